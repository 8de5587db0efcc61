"""Rotors: ``compile_bivector`` / ``apply_rotor`` with autograd to both the
bivector and x (reference algebra.py:343-373, eigh_exp.py, givens_factor.py,
givens_apply/mb_perm_packed.py).

The compiled rotor ``cs`` is an opaque fp32 tensor: the per-grade blade-minor
matrices of Rm = expm(2 (M - M^T)). ``apply_rotor(cs, x)`` evaluates
y_k = x_k C_k per grade, which equals the reference's Givens-chain sandwich
R~ x R. Unlike the reference (mb_perm_packed.py:42), x receives a gradient.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


def _sizes(n):
    a, b = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(_lib.load().cb_rotor_sizes(n, ctypes.byref(a), ctypes.byref(b)), "cb_rotor_sizes")
    return a.value, b.value


class _CompileFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, bivector, n):
        cs_n, st_n = _sizes(n)
        beta = bivector.detach().contiguous()
        cs = torch.empty(cs_n, device=beta.device, dtype=torch.float32)
        state = torch.empty(st_n, device=beta.device, dtype=torch.float64)
        with torch.cuda.device(beta.device):
            st = _lib.load().cb_rotor_compile(_lib.ptr(beta), n, _lib.ptr(cs), _lib.ptr(state),
                                              _lib.stream_of(beta))
        _lib.check(st, "cb_rotor_compile")
        ctx.save_for_backward(state)
        ctx.n = n
        ctx.shape = bivector.shape
        return cs

    @staticmethod
    def backward(ctx, dcs):
        (state,) = ctx.saved_tensors
        dcs = dcs.contiguous().float()
        nb = ctx.n * (ctx.n - 1) // 2
        dbeta = torch.empty(nb, device=dcs.device, dtype=torch.float32)
        with torch.cuda.device(dcs.device):
            st = _lib.load().cb_rotor_compile_bwd(_lib.ptr(state), _lib.ptr(dcs), ctx.n,
                                                  _lib.ptr(dbeta), _lib.stream_of(dcs))
        _lib.check(st, "cb_rotor_compile_bwd")
        return dbeta.view(ctx.shape), None


def _apply_raw(cs, x, n, transpose=False):
    y = torch.empty_like(x)
    with torch.cuda.device(x.device):
        st = _lib.load().cb_rotor_apply(_lib.ptr(cs), _lib.ptr(x), _lib.ptr(y), x.shape[0], n,
                                        1 if transpose else 0, _lib.stream_of(x))
    _lib.check(st, "cb_rotor_apply")
    return y


def _aligned(t):
    """Contiguous with 16-byte aligned rows (the n = 7, 8 kernels read rows
    through TMA); offset views are copied."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


class _ApplyFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cs, x, n):
        cs = cs.contiguous()
        x = _aligned(x)
        ctx.save_for_backward(cs, x)
        ctx.n = n
        return _apply_raw(cs, x, n)

    @staticmethod
    def backward(ctx, g):
        cs, x = ctx.saved_tensors
        n = ctx.n
        g = _aligned(g)
        need_cs, need_x = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dx = torch.empty_like(x) if need_x else None
        dcs = None
        if need_cs:
            lib = _lib.load()
            with torch.cuda.device(g.device):
                wb = ctypes.c_int64()
                _lib.check(lib.cb_rotor_workspace_bytes(n, x.shape[0], ctypes.byref(wb)),
                           "cb_rotor_workspace_bytes")
                ws = torch.empty(max(wb.value, 1), device=g.device, dtype=torch.uint8)
                dcs = torch.empty_like(cs)
                st = lib.cb_rotor_apply_bwd(_lib.ptr(cs), _lib.ptr(x), _lib.ptr(g), _lib.ptr(dx),
                                            _lib.ptr(dcs), x.shape[0], n, _lib.ptr(ws),
                                            wb.value, _lib.stream_of(g))
            _lib.check(st, "cb_rotor_apply_bwd")
        elif need_x:
            dx = _apply_raw(cs, g, n, transpose=True)
        return dcs, dx, None


class RotorEngine:
    """Per-algebra rotor front end used by CliffordAlgebra."""

    def __init__(self, n, device):
        if not 2 <= n <= 10:
            raise ValueError(f"rotor path supports 2 <= n <= 10; got n={n}")
        self.n = n
        self.device = device
        self.cs_floats, self.state_doubles = _sizes(n)

    def compile(self, bivector):
        return _CompileFn.apply(bivector, self.n)

    def apply(self, cs, x):
        if not isinstance(cs, torch.Tensor) or cs.numel() != self.cs_floats or \
                cs.dtype != torch.float32 or cs.device != x.device:
            raise ValueError(
                f"cs must be a compiled rotor for n={self.n} (float32, {self.cs_floats} "
                f"entries, on {x.device}); got {type(cs).__name__}")
        return _ApplyFn.apply(cs, x, self.n)
