"""Batch-by-batch multivector products with autograd.

Same free functions, argument order and defaults as the reference
(``src/cliffordcuda/__init__.py:2-21``): ``geom_prod``, ``wedge_prod``,
``inner_prod``, ``left_contract``, ``right_contract``, ``regressive_prod``,
each ``f(a, b, metric=None)`` on ``(batch, 2^n)`` fp32 CUDA tensors in
bit-pattern blade order, ``metric=None`` meaning Cl(n, 0).

Forward and backward each call the native library once
(``cb_bilinear`` / ``cb_bilinear_bwd``); there are no lookup tables: the
metric travels as two bitmasks. Backward sums (reference
``extensions/ga/geom_prod.py:241-250``):

    grad_a[k] = sum_i s(k, i) * b[i] * g[k ^ i]
    grad_b[k] = sum_i s(i, k) * a[i] * g[k ^ i]
"""
from __future__ import annotations

import torch

from . import _lib


def _normalize_metric(n, metric):
    """Length-n tuple of {-1, 0, 1}; None -> Cl(n, 0)
    (reference extensions/ga/geom_prod.py:32-41)."""
    if metric is None:
        return (1,) * n
    metric = tuple(int(m) for m in metric)
    if len(metric) != n:
        raise ValueError(f"metric must have {n} entries, got {len(metric)}")
    if any(m not in (-1, 0, 1) for m in metric):
        raise ValueError(f"metric entries must be in {{-1, 0, 1}}, got {metric}")
    return metric


def metric_masks(metric):
    """(neg_mask, zero_mask): bit t set when generator t squares to -1 / 0."""
    neg = sum(1 << t for t, m in enumerate(metric) if m == -1)
    zero = sum(1 << t for t, m in enumerate(metric) if m == 0)
    return neg, zero


def _dims(a, b):
    if not (isinstance(a, torch.Tensor) and isinstance(b, torch.Tensor)):
        raise ValueError("a and b must be torch.Tensors")
    if a.dim() != 2 or b.dim() != 2 or a.shape != b.shape:
        raise ValueError(
            f"a and b must be 2D (batch, 2^n) of equal shape; got {tuple(a.shape)} "
            f"and {tuple(b.shape)}")
    dim = a.size(-1)
    n = dim.bit_length() - 1
    if (1 << n) != dim:
        raise ValueError(f"dim must be a power of two, got {dim}")
    if n < 5:
        raise ValueError("n>=5 required; lower n is not supported by this kernel layout")
    if not (a.is_cuda and b.is_cuda) or a.device != b.device:
        raise ValueError(f"a and b must be CUDA tensors on one device; got {a.device}, {b.device}")
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError(f"a and b must be float32; got {a.dtype}, {b.dtype}")
    return n


def bilinear_raw(op, mode, x, y, n, metric, out=None, direct=False):
    """One native bilinear sum (no autograd). x, y contiguous fp32 CUDA.
    direct=True always uses the blade-by-blade kernels (cb_bilinear_direct)."""
    neg, zero = metric_masks(metric)
    if out is None:
        out = torch.empty_like(x)
    lib = _lib.load()
    fn = lib.cb_bilinear_direct if direct else lib.cb_bilinear
    with torch.cuda.device(x.device):
        st = fn(_lib.OPS[op], _lib.MODES[mode], _lib.ptr(x), _lib.ptr(y),
                _lib.ptr(out), x.shape[0], n, neg, zero, _lib.stream_of(x))
    _lib.check(st, f"cb_bilinear({op}, {mode})")
    return out


def bilinear_bwd_raw(op, a, b, g, n, metric, ga=None, gb=None):
    """Both backward sums of product `op` (no autograd) into ga / gb; either
    may be None to skip it. a, b, g contiguous fp32 CUDA."""
    neg, zero = metric_masks(metric)
    lib = _lib.load()
    with torch.cuda.device(g.device):
        st = lib.cb_bilinear_bwd(_lib.OPS[op], _lib.ptr(a), _lib.ptr(b), _lib.ptr(g),
                                 _lib.ptr(ga), _lib.ptr(gb), a.shape[0], n, neg, zero,
                                 _lib.stream_of(g))
    _lib.check(st, f"cb_bilinear_bwd({op})")
    return ga, gb


class _BilinearFunc(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, op, n, metric):
        ctx.save_for_backward(a, b)
        ctx.op, ctx.n, ctx.metric = op, n, metric
        return bilinear_raw(op, "fwd", a, b, n, metric)

    @staticmethod
    def backward(ctx, grad_c):
        a, b = ctx.saved_tensors
        g = grad_c.contiguous()
        need_a, need_b = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        ga = torch.empty_like(a) if need_a else None
        gb = torch.empty_like(b) if need_b else None
        if need_a or need_b:
            bilinear_bwd_raw(ctx.op, a, b, g, ctx.n, ctx.metric, ga, gb)
        return ga, gb, None, None, None


def _product(op, a, b, metric):
    n = _dims(a, b)
    metric = _normalize_metric(n, metric)
    if op == "reg" and 0 in metric:
        raise ValueError(
            "regressive_prod is undefined for degenerate metrics "
            "(any 0 in the metric makes the pseudoscalar non-invertible).")
    return _BilinearFunc.apply(a.contiguous(), b.contiguous(), op, n, metric)


def geom_prod(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Geometric product a b in Cl(p, q, r) (reference geom_prod.py:253-276)."""
    return _product("gp", a, b, metric)


def wedge_prod(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Outer product a ^ b: terms with disjoint blades (wedge_prod/chunk.py:105-121)."""
    return _product("wedge", a, b, metric)


def inner_prod(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Hestenes inner product, scalars included: terms with i subset j or
    j subset i (inner_prod/chunk.py:101-115)."""
    return _product("inner", a, b, metric)


def left_contract(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Left contraction: terms with i subset j (left_contract.py:121-138)."""
    return _product("lc", a, b, metric)


def right_contract(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Right contraction: terms with j subset i (right_contract.py:76-127)."""
    return _product("rc", a, b, metric)


def regressive_prod(a: torch.Tensor, b: torch.Tensor, metric=None) -> torch.Tensor:
    """Regressive product dual(dual(a) ^ dual(b)), non-degenerate metrics only
    (regressive_prod.py:186-201; _einsum_refs.py:86-124)."""
    return _product("reg", a, b, metric)
