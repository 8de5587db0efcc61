"""Per-blade maps and the squared norm on the native kernels, with autograd.

reverse / grade_involution / clifford_conjugation / grade_projection / dual
multiply every coefficient by a per-blade factor (the dual also reverses the
coefficient order); norm_sq reduces each row. The reference computed these as
torch elementwise multiplies by cached sign vectors
(src/cliffordcuda/algebra.py:195-336); here each is one pass of
``cb_blade_map`` / ``cb_norm_sq``. Backward: the maps are linear, so the
gradient is the transposed map (itself for the diagonal ones, CB_MAP_DUAL_T
for the dual); norm_sq's is 2 w x g.
"""
from __future__ import annotations

import torch

from . import _lib
from .products import metric_masks

_TRANSPOSE = {"reverse": "reverse", "involute": "involute", "conjugate": "conjugate",
              "grade": "grade", "dual": "dual_t", "dual_t": "dual"}


def _n_of(x):
    dim = x.shape[-1]
    n = dim.bit_length() - 1
    if (1 << n) != dim or n < 1:
        raise ValueError(f"dim must be a power of two >= 2, got {dim}")
    return n


def map_raw(kind, x, n, metric, grade=0):
    """One native blade map (no autograd) on a contiguous 2-D fp32 CUDA tensor."""
    neg, zero = metric_masks(metric)
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        st = _lib.load().cb_blade_map(_lib.MAPS[kind], _lib.ptr(x), _lib.ptr(out), x.shape[0], n,
                                      neg, zero, grade, _lib.stream_of(x))
    _lib.check(st, f"cb_blade_map({kind})")
    return out


class _MapFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kind, n, metric, grade):
        ctx.args = (kind, n, metric, grade)
        return map_raw(kind, x, n, metric, grade)

    @staticmethod
    def backward(ctx, g):
        kind, n, metric, grade = ctx.args
        return map_raw(_TRANSPOSE[kind], g.contiguous(), n, metric, grade), None, None, None, None


class _NormSqFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, n, metric):
        ctx.save_for_backward(x)
        ctx.args = (n, metric)
        neg, zero = metric_masks(metric)
        out = torch.empty(x.shape[0], device=x.device, dtype=x.dtype)
        with torch.cuda.device(x.device):
            st = _lib.load().cb_norm_sq(_lib.ptr(x), _lib.ptr(out), x.shape[0], n, neg, zero,
                                        _lib.stream_of(x))
        _lib.check(st, "cb_norm_sq")
        return out

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        n, metric = ctx.args
        neg, zero = metric_masks(metric)
        g = g.contiguous()
        dx = torch.empty_like(x)
        with torch.cuda.device(x.device):
            st = _lib.load().cb_norm_sq_bwd(_lib.ptr(x), _lib.ptr(g), _lib.ptr(dx), x.shape[0], n,
                                            neg, zero, _lib.stream_of(x))
        _lib.check(st, "cb_norm_sq_bwd")
        return dx, None, None


def _rows(x, n):
    return x.reshape(-1, 1 << n).contiguous()


def blade_map(kind, x, metric, grade=0):
    """map `kind` over the last axis of x (any leading shape)."""
    n = _n_of(x)
    y = _MapFn.apply(_rows(x, n), kind, n, tuple(metric), grade)
    return y.view(x.shape)


def norm_sq(x, metric):
    """<x x~>_0 per multivector: shape x.shape[:-1]."""
    n = _n_of(x)
    return _NormSqFn.apply(_rows(x, n), n, tuple(metric)).view(x.shape[:-1])


def reverse(x):
    """Reversion x~ of (..., 2^n) multivectors: grade k -> (-1)^(k(k-1)/2)
    (reference extensions/ga/inverse.py:64-67; the metric is not used)."""
    n = _n_of(x)
    return blade_map("reverse", x, (1,) * n)
