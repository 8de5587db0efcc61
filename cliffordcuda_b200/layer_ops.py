"""Shared-weight product layers: y = op(x, w) with one weight row for the
whole batch (reference layers.py:43-47, which materialised w.expand_as(x)
and ran the batch-by-batch kernel, then let autograd sum the per-row weight
gradients).

The GeometricProductLayer of Euclidean Cl(8,0) runs through the algebra's
real 16 x 16 matrix representation (cb_layer_gp8_*): one 16 x 16 product per
row with the fixed matrix rho(w). Other layers with n = 7 and 8 run as a
dense contraction on the tensor cores:
M(w) is assembled once per call (cb_layer_prepare), the forward is the
3xTF32 GEMM y = x M, and the backward gives dx = dy M^T and the weight
gradient folded from G = x^T dy (cb_layer_backward). Other n run the
batch-by-batch kernel with the weight broadcast, as the reference did.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from . import products as _p

GEMM_N = (7, 8)


def _aligned(t):
    """Contiguous with 16-byte aligned rows (the layer kernels stream rows with
    TMA / bulk copies); offset views are copied."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _workspace(n, batch, device):
    wb = ctypes.c_int64()
    _lib.check(_lib.load().cb_layer_workspace_bytes(n, batch, ctypes.byref(wb)),
               "cb_layer_workspace_bytes")
    return torch.empty(max(wb.value, 4), device=device, dtype=torch.uint8)


def prepare(op, weight, n, metric):
    """mats = [M^T hi | M^T lo | M hi | M lo] for the current weight."""
    neg, zero = _p.metric_masks(metric)
    D = 1 << n
    w = weight.detach().contiguous().view(-1)
    mats = torch.empty(4 * D * D, device=w.device, dtype=torch.float32)
    ws = _workspace(n, 1, w.device)
    with torch.cuda.device(w.device):
        st = _lib.load().cb_layer_prepare(_lib.OPS[op], _lib.ptr(w), n, neg, zero, _lib.ptr(mats),
                                          _lib.ptr(ws), ws.numel(), _lib.stream_of(w))
    _lib.check(st, "cb_layer_prepare")
    return mats


class _LayerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, op, n, metric):
        mats = prepare(op, weight, n, metric)
        y = torch.empty_like(x)
        with torch.cuda.device(x.device):
            st = _lib.load().cb_layer_forward(_lib.ptr(mats), _lib.ptr(x), _lib.ptr(y),
                                              x.shape[0], n, _lib.stream_of(x))
        _lib.check(st, "cb_layer_forward")
        ctx.save_for_backward(x, mats)
        ctx.op, ctx.n, ctx.metric, ctx.wshape = op, n, metric, weight.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x, mats = ctx.saved_tensors
        dy = _aligned(dy)
        need_x, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dx = torch.empty_like(x) if need_x else None
        dw = torch.empty(1 << ctx.n, device=x.device, dtype=torch.float32) if need_w else None
        if need_x or need_w:
            neg, zero = _p.metric_masks(ctx.metric)
            ws = _workspace(ctx.n, x.shape[0], x.device)
            with torch.cuda.device(x.device):
                st = _lib.load().cb_layer_backward(
                    _lib.OPS[ctx.op], _lib.ptr(mats), _lib.ptr(x), _lib.ptr(dy), _lib.ptr(dx),
                    _lib.ptr(dw), x.shape[0], ctx.n, neg, zero, _lib.ptr(ws), ws.numel(),
                    _lib.stream_of(x))
            _lib.check(st, "cb_layer_backward")
        return dx, (dw.view(ctx.wshape) if dw is not None else None), None, None, None


class _Gp8LayerFn(torch.autograd.Function):
    """GeometricProductLayer of Cl(8,0) through the 16 x 16 matrix
    representation (cb_layer_gp8_*): rho(y) = rho(x) rho(w)."""

    @staticmethod
    def forward(ctx, x, weight):
        w = weight.detach().contiguous().view(-1)
        mats = torch.empty(1024, device=x.device, dtype=torch.float32)
        y = torch.empty_like(x)
        lib = _lib.load()
        with torch.cuda.device(x.device):
            st = lib.cb_layer_gp8_prepare(_lib.ptr(w), _lib.ptr(mats), _lib.stream_of(x))
            _lib.check(st, "cb_layer_gp8_prepare")
            st = lib.cb_layer_gp8_forward(_lib.ptr(mats), _lib.ptr(x), _lib.ptr(y), x.shape[0],
                                          _lib.stream_of(x))
        _lib.check(st, "cb_layer_gp8_forward")
        ctx.save_for_backward(x, mats)
        ctx.wshape = weight.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x, mats = ctx.saved_tensors
        dy = _aligned(dy)
        need_x, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dx = torch.empty_like(x) if need_x else None
        dw = torch.empty(256, device=x.device, dtype=torch.float32) if need_w else None
        if need_x or need_w:
            ws = _workspace(8, x.shape[0], x.device)
            with torch.cuda.device(x.device):
                st = _lib.load().cb_layer_gp8_backward(
                    _lib.ptr(mats), _lib.ptr(x), _lib.ptr(dy), _lib.ptr(dx), _lib.ptr(dw),
                    x.shape[0], _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
            _lib.check(st, "cb_layer_gp8_backward")
        return dx, (dw.view(ctx.wshape) if dw is not None else None)


def layer_product(op, x, weight, n, metric):
    if op == "gp" and n == 8 and all(m == 1 for m in metric):
        return _Gp8LayerFn.apply(_aligned(x), weight)
    if n in GEMM_N:
        return _LayerFn.apply(_aligned(x), weight, op, n, tuple(metric))
    w = weight.expand_as(x).contiguous()
    return _p._product(op, x, w, metric)
