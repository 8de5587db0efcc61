"""Parity at the BASELINE configs' own shapes, where split-K partial counts,
fp64 reductions and sparse rows actually matter.

* config 3: the product layers at 524,288 rows (the per-GPU share of
  4,194,304 over 8 GPUs): the GeometricProductLayer on both routes (16 x 16
  matrix representation and dense 3xTF32 tcgen05 GEMM), the Wedge and
  LeftContraction layers (tcgen05 GEMM). y and dx on sampled rows against
  the oracle; dw against the oracle's weight gradient folded from the fp64
  G = x^T dy of the whole batch on the CPU (layers.py:43-47 semantics);
* config 4: the rotor at 2,097,152 rows in Cl(7,1), training mode: y and dx
  on sampled rows against the C oracle's blade-minor matrix; dbeta against
  fp64 autograd of the compile map at G = x^T g, with G from a CPU fp64 GEMM
  on a 131,072-row call and from an fp64 cuBLAS GEMM at full size;
* config 5: Cl(9,0,1) with 10% of the rows restricted to grades 0/2/4 (the
  bench's construction): sampled even-versor and dense rows against the
  oracle, and the odd grades of an even-versor product exactly zero.
Tolerance: relative L2 <= 1e-5 against float64 (tests/helpers.py).
"""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib, layer_ops
from cliffordcuda_b200.products import bilinear_raw
from oracle import ga_oracle as O
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _sample(batch, k, seed):
    return torch.randperm(batch, generator=torch.Generator().manual_seed(seed))[:k].to(DEV)


def _G_cpu(x, y):
    """sum over rows of x^T y in float64 on the CPU."""
    return x.detach().cpu().double().T @ y.detach().cpu().double()


@pytest.mark.parametrize("route", ["gp_matrix", "gp_dense", "wedge", "lc"])
def test_layer_config3_shape(route):
    batch, n, metric = 524_288, 8, (1,) * 8
    op = route.split("_")[0]
    gen = torch.Generator(device=DEV).manual_seed(31)
    x = torch.randn(batch, 256, device=DEV, generator=gen)
    dy = torch.randn(batch, 256, device=DEV, generator=gen)
    w = torch.randn(1, 256, device=DEV, generator=gen) / 16
    cl = cc.CliffordAlgebra(list(metric), device=DEV)
    xr = x.clone().requires_grad_(True)
    if route == "gp_dense":     # the tcgen05 route of the GP layer, forced
        wt = w.clone().requires_grad_(True)
        y = layer_ops._LayerFn.apply(xr, wt, "gp", n, metric)
        y.backward(dy)
        dw = wt.grad
    else:
        cls = {"gp": cc.GeometricProductLayer, "wedge": cc.WedgeProductLayer,
               "lc": cc.LeftContractionLayer}[op]
        layer = cls(cl)
        with torch.no_grad():
            layer.weight.copy_(w)
        y = layer(xr)
        y.backward(dy)
        dw = layer.weight.grad
    rows = _sample(batch, 64, 5)
    wn = w.cpu().numpy().ravel()
    wrep = np.repeat(wn.reshape(1, -1), 64, axis=0)
    ref_y, ref_dx, _ = O.forward_backward(op, n, metric, x[rows].cpu().numpy(), wrep,
                                          dy[rows].cpu().numpy())
    assert rel_l2(y[rows].detach().cpu().numpy(), ref_y) <= REL_L2_TOL
    assert rel_l2(xr.grad[rows].cpu().numpy(), ref_dx) <= REL_L2_TOL
    dw_ref = O.layer_dw_from_G(op, n, metric, _G_cpu(x, dy).numpy())
    err = rel_l2(dw.cpu().numpy().ravel(), dw_ref)
    assert err <= REL_L2_TOL, f"{route} dw: rel L2 {err:.3e}"
    _lib.device_status(DEV)


def _rotor_step(cl, beta, x, g):
    bt = beta.clone().requires_grad_(True)
    xt = x.clone().requires_grad_(True)
    y = cl.apply_bivector(bt, xt)
    y.backward(g)
    return y.detach(), xt.grad, bt.grad


def test_rotor_config4_shape_gradients():
    n, batch, metric = 8, 2_097_152, [1] * 7 + [-1]
    gen = torch.Generator(device=DEV).manual_seed(41)
    x = torch.randn(batch, 256, device=DEV, generator=gen)
    g = torch.randn(batch, 256, device=DEV, generator=gen)
    beta = 0.1 * torch.randn(1, 28, device=DEV, generator=gen)
    cl = cc.CliffordAlgebra(metric, device=DEV)
    beta_np = beta.cpu().numpy().ravel().astype(np.float64)
    C = O.rotor_blade_matrix(n, O.rotor_matrix(n, beta_np))

    # a 131,072-row call: G from a CPU fp64 GEMM
    sl = 131_072
    y, dx, db = _rotor_step(cl, beta, x[:sl], g[:sl])
    db_ref = O.rotor_dbeta_from_G(n, beta_np, _G_cpu(x[:sl], g[:sl]).numpy())
    assert rel_l2(db.cpu().numpy().ravel(), db_ref) <= REL_L2_TOL

    # the full config-4 batch
    y, dx, db = _rotor_step(cl, beta, x, g)
    rows = _sample(batch, 64, 6)
    xs, gs = x[rows].cpu().double().numpy(), g[rows].cpu().double().numpy()
    assert rel_l2(y[rows].cpu().numpy(), xs @ C) <= REL_L2_TOL
    assert rel_l2(dx[rows].cpu().numpy(), gs @ C.T) <= REL_L2_TOL
    G = (x.double().T @ g.double()).cpu().numpy()     # fp64 cuBLAS, not this library
    db_ref = O.rotor_dbeta_from_G(n, beta_np, G)
    err = rel_l2(db.cpu().numpy().ravel(), db_ref)
    assert err <= REL_L2_TOL, f"dbeta at 2M rows: rel L2 {err:.3e}"
    _lib.device_status(DEV)


@pytest.mark.parametrize("op", ["gp", "lc"])
def test_config5_even_versor_rows(op):
    """Cl(9,0,1), 131,072 rows, 10% restricted to grades 0/2/4 exactly as the
    config-5 bench builds them."""
    n, metric, batch = 10, (1,) * 9 + (0,), 131_072
    D = 1 << n
    gen = torch.Generator(device=DEV).manual_seed(5)
    a, b, g = (torch.randn(batch, D, device=DEV, generator=gen) for _ in range(3))
    grades = torch.tensor([bin(i).count("1") for i in range(D)], device=DEV)
    even = ((grades == 0) | (grades == 2) | (grades == 4)).float()
    sparse = torch.randperm(batch, generator=torch.Generator().manual_seed(9))[: batch // 10]
    sparse = sparse.to(DEV)
    a[sparse] *= even
    b[sparse] *= even
    is_sparse = torch.zeros(batch, dtype=torch.bool, device=DEV)
    is_sparse[sparse] = True
    dense = torch.nonzero(~is_sparse).view(-1)
    rows = torch.cat([sparse[:32], dense[_sample(dense.numel(), 32, 3)]])
    for mode, x, y in (("fwd", a, b), ("grad_a", b, g), ("grad_b", a, g)):
        out = bilinear_raw(op, mode, x, y, n, metric)
        ref = O.product(op, mode, n, metric, x[rows].cpu().numpy(), y[rows].cpu().numpy())
        err = rel_l2(out[rows].cpu().numpy(), ref)
        assert err <= REL_L2_TOL, f"{op} {mode}: rel L2 {err:.3e}"
        if mode == "fwd" and op == "gp":
            # an even versor times an even versor is even: the odd grades of
            # those rows vanish (to fp32 rounding on the matrix-representation route)
            odd = (grades % 2 == 1)
            ev = out[sparse]
            assert ev[:, odd].abs().max().item() <= 1e-5 * ev.abs().max().item()
        del out
    _lib.device_status(DEV)
