"""Product layers (GEMM path for n = 7, 8; batch-by-batch kernel otherwise)
against the oracle: y = op(x, w), dx, and dw = sum over the batch of the
second-operand gradient, as the reference's expand_as formulation gives
(layers.py:43-47)."""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib
from oracle import ga_oracle as O
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

LAYERS = {"gp": cc.GeometricProductLayer, "wedge": cc.WedgeProductLayer,
          "inner": cc.InnerProductLayer, "lc": cc.LeftContractionLayer,
          "rc": cc.RightContractionLayer, "reg": cc.RegressiveProductLayer}


def oracle_layer(op, n, metric, x, w, g):
    wrep = np.repeat(w.reshape(1, -1), x.shape[0], axis=0)
    y, dx, dwr = O.forward_backward(op, n, metric, x, wrep, g)
    return y, dx, dwr.sum(axis=0)


def run_layer(op, metric, x, w, g):
    cl = cc.CliffordAlgebra(list(metric), device=DEV)
    layer = LAYERS[op](cl)
    with torch.no_grad():
        layer.weight.copy_(torch.tensor(w, device=DEV).view(1, -1))
    xt = torch.tensor(x, device=DEV, requires_grad=True)
    y = layer(xt)
    y.backward(torch.tensor(g, device=DEV))
    return (y.detach().cpu().numpy(), xt.grad.cpu().numpy(),
            layer.weight.grad.cpu().numpy().ravel())


@pytest.mark.parametrize("op", ["gp"])
def test_gemm_layer_forward_small(op):
    n, metric = 8, (1,) * 8
    rng = np.random.default_rng(0)
    x = rng.standard_normal((256, 256)).astype(np.float32)
    w = (rng.standard_normal(256) / 16).astype(np.float32)
    cl = cc.CliffordAlgebra(list(metric), device=DEV)
    layer = LAYERS[op](cl)
    with torch.no_grad():
        layer.weight.copy_(torch.tensor(w, device=DEV).view(1, -1))
        y = layer(torch.tensor(x, device=DEV)).cpu().numpy()
    ref = oracle_layer(op, n, metric, x, w, np.zeros_like(x))[0]
    assert rel_l2(y, ref) <= REL_L2_TOL


@pytest.mark.parametrize("op", list(LAYERS))
@pytest.mark.parametrize("n,metric", [(8, (1,) * 8), (8, (1,) * 7 + (-1,)),
                                      (7, (1,) * 6 + (-1,)), (7, (1,) * 6 + (0,)),
                                      (5, (1, 1, -1, -1, 1)), (6, (1,) * 6)])
def test_layer_fwd_bwd(op, n, metric):
    if op == "reg" and 0 in metric:
        pytest.skip("regressive undefined for degenerate metrics")
    rng = np.random.default_rng(n * 13 + list(LAYERS).index(op))
    batch = 1000 + 37
    D = 1 << n
    x = rng.standard_normal((batch, D)).astype(np.float32)
    g = rng.standard_normal((batch, D)).astype(np.float32)
    w = (rng.standard_normal(D) / np.sqrt(D)).astype(np.float32)
    got = run_layer(op, metric, x, w, g)
    ref = oracle_layer(op, n, metric, x, w, g)
    for name, a, b in zip(("y", "dx", "dw"), got, ref):
        assert rel_l2(a, b) <= REL_L2_TOL, f"{op} n={n} {metric} {name}: {rel_l2(a, b):.3e}"


@pytest.mark.parametrize("batch", [1, 127, 129, 4096 + 5])
def test_layer_ragged_batches(batch):
    n, metric = 8, (1,) * 8
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, 256)).astype(np.float32)
    g = rng.standard_normal((batch, 256)).astype(np.float32)
    w = (rng.standard_normal(256) / 16).astype(np.float32)
    got = run_layer("gp", metric, x, w, g)
    ref = oracle_layer("gp", n, metric, x, w, g)
    for a, b in zip(got, ref):
        assert rel_l2(a, b) <= REL_L2_TOL


@pytest.mark.parametrize("batch", [5, 1037])
def test_gp8_routes_agree(batch):
    """The GeometricProductLayer of Cl(8,0) runs through the 16 x 16 matrix
    representation (cb_layer_gp8_*); the dense tcgen05 route (cb_layer_*)
    stays reachable. Both against the oracle and against each other."""
    from cliffordcuda_b200 import layer_ops
    n, metric = 8, (1,) * 8
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, 256)).astype(np.float32)
    g = rng.standard_normal((batch, 256)).astype(np.float32)
    w = (rng.standard_normal(256) / 16).astype(np.float32)
    ref = oracle_layer("gp", n, metric, x, w, g)
    outs = []
    for dense in (False, True):
        wt = torch.tensor(w, device=DEV).view(1, -1).requires_grad_(True)
        xt = torch.tensor(x, device=DEV, requires_grad=True)
        if dense:
            y = layer_ops._LayerFn.apply(xt, wt, "gp", n, metric)
        else:
            y = layer_ops.layer_product("gp", xt, wt, n, metric)
        y.backward(torch.tensor(g, device=DEV))
        got = (y.detach().cpu().numpy(), xt.grad.cpu().numpy(), wt.grad.cpu().numpy().ravel())
        for name, a, b in zip(("y", "dx", "dw"), got, ref):
            assert rel_l2(a, b) <= REL_L2_TOL, f"dense={dense} {name}: {rel_l2(a, b):.3e}"
        outs.append(got)
    for a, b in zip(*outs):
        assert rel_l2(a, b) < 1e-5


@pytest.mark.parametrize("op,metric", [("gp", (1,) * 8), ("wedge", (1,) * 8),
                                       ("lc", (1,) * 7 + (-1,))])
def test_layer_unaligned_views(op, metric):
    """x and the upstream gradient as views starting one float into their
    buffers: the layer copies them to aligned rows and matches the oracle."""
    n, batch = 8, 37
    rng = np.random.default_rng(11)
    x = rng.standard_normal((batch, 256)).astype(np.float32)
    g = rng.standard_normal((batch, 256)).astype(np.float32)
    w = (rng.standard_normal(256) / 16).astype(np.float32)
    ref = oracle_layer(op, n, metric, x, w, g)
    bx = torch.zeros(batch * 256 + 1, device=DEV)
    bx[1:].copy_(torch.from_numpy(x).view(-1))
    xt = bx[1:].view(batch, 256).requires_grad_(True)
    bg = torch.zeros(batch * 256 + 1, device=DEV)
    bg[1:].copy_(torch.from_numpy(g).view(-1))
    cl = cc.CliffordAlgebra(list(metric), device=DEV)
    layer = LAYERS[op](cl)
    with torch.no_grad():
        layer.weight.copy_(torch.tensor(w, device=DEV).view(1, -1))
    y = layer(xt)
    y.backward(bg[1:].view(batch, 256))
    got = (y.detach().cpu().numpy(), xt.grad.cpu().numpy(), layer.weight.grad.cpu().numpy().ravel())
    for name, a, b in zip(("y", "dx", "dw"), got, ref):
        assert rel_l2(a, b) <= REL_L2_TOL, f"{op} {name}: {rel_l2(a, b):.3e}"
