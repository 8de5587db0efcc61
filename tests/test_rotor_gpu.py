"""Rotor path (compile_bivector / apply_rotor / RotorLayer) against the oracle.

* forward against the golden sandwich computed with the reference's EinsumGP;
* forward at n = 7..10 (fast kernels for 7, 8; generic for 9, 10) against the
  C oracle (blade minors of Rm = expm(2 (M - M^T)));
* gradients to x and to the bivector against float64 autograd of the same
  map (torch.linalg.matrix_exp + determinants);
* at BASELINE config 4's shape: sampled rows and per-row norm preservation
  (Rm is orthogonal, so the outermorphism is an isometry of the blades).
"""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib
from oracle import ga_oracle as O
from tests.helpers import REL_L2_TOL, load_npz, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def algebra(n, metric=None):
    return cc.CliffordAlgebra(metric or [1] * n, device=DEV)


@pytest.mark.parametrize("n", [7, 8])
def test_golden_sandwich(n):
    R = load_npz("rotor.npz")
    cl = algebra(n)
    beta = torch.tensor(R[f"{n}|beta"], device=DEV).view(1, -1)
    x = torch.tensor(R[f"{n}|x"], device=DEV)
    y = cl.apply_bivector(beta, x)
    assert rel_l2(y.detach().cpu().numpy(), R[f"{n}|y"]) <= REL_L2_TOL


@pytest.mark.parametrize("n,scale,batch", [(7, 0.1, 100), (8, 0.1, 77), (8, 1.0, 64),
                                           (9, 0.3, 9), (10, 0.3, 3)])
def test_forward_vs_oracle(n, scale, batch):
    rng = np.random.default_rng(n * 7 + batch)
    beta = (scale * rng.standard_normal(n * (n - 1) // 2)).astype(np.float32)
    x = rng.standard_normal((batch, 1 << n)).astype(np.float32)
    cl = algebra(n)
    with torch.no_grad():
        cs = cl.compile_bivector(torch.tensor(beta, device=DEV).view(1, -1))
        y = cl.apply_rotor(cs, torch.tensor(x, device=DEV))
    ref = O.rotor_apply(n, beta, x)
    assert rel_l2(y.cpu().numpy(), ref) <= REL_L2_TOL


def test_metric_is_ignored_like_reference():
    """Cl(7,1): the reference's rotor path never reads the metric."""
    rng = np.random.default_rng(4)
    beta = torch.tensor(0.1 * rng.standard_normal((1, 28)), device=DEV, dtype=torch.float32)
    x = torch.randn(16, 256, device=DEV)
    y1 = algebra(8).apply_bivector(beta, x)
    y2 = algebra(8, [1] * 7 + [-1]).apply_bivector(beta, x)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("n,batch", [(7, 50), (8, 33), (9, 5)])
def test_gradients_vs_fp64_autograd(n, batch):
    rng = np.random.default_rng(100 + n)
    beta = (0.2 * rng.standard_normal(n * (n - 1) // 2)).astype(np.float32)
    x = rng.standard_normal((batch, 1 << n)).astype(np.float32)
    g = rng.standard_normal((batch, 1 << n)).astype(np.float32)
    y_ref, dx_ref, db_ref = O.rotor_grads_torch(n, beta, x, g)
    cl = algebra(n)
    bt = torch.tensor(beta, device=DEV).view(1, -1).requires_grad_(True)
    xt = torch.tensor(x, device=DEV, requires_grad=True)
    y = cl.apply_bivector(bt, xt)
    y.backward(torch.tensor(g, device=DEV))
    assert rel_l2(y.detach().cpu().numpy(), y_ref) <= REL_L2_TOL
    assert rel_l2(xt.grad.cpu().numpy(), dx_ref) <= REL_L2_TOL
    assert rel_l2(bt.grad.cpu().numpy().ravel(), db_ref) <= 1e-4


def test_rotor_layer_train_and_eval():
    cl = algebra(8, [1] * 7 + [-1])
    layer = cc.RotorLayer(cl)
    with torch.no_grad():
        layer.bivector.mul_(0.1)
    x = torch.randn(40, 256, device=DEV)
    layer.train()
    y_train = layer(x)
    y_train.sum().backward()
    assert layer.bivector.grad is not None and torch.isfinite(layer.bivector.grad).all()
    layer.eval()
    y_eval = layer(x)
    assert layer._cs is not None
    assert torch.allclose(y_train.detach(), y_eval, atol=1e-5)
    ref = O.rotor_apply(8, layer.bivector.detach().cpu().numpy().ravel(), x.cpu().numpy())
    assert rel_l2(y_eval.cpu().numpy(), ref) <= REL_L2_TOL


def test_rotor_boundary_errors():
    with pytest.raises(ValueError):
        algebra(6).compile_bivector(torch.zeros(1, 15, device=DEV))
    cl = algebra(8)
    with pytest.raises(ValueError):
        cl.compile_bivector(torch.zeros(2, 28, device=DEV))
    with pytest.raises(ValueError):
        cl.compile_bivector(torch.zeros(1, 27, device=DEV))
    with pytest.raises(ValueError):
        cl.apply_rotor(torch.zeros(5, device=DEV), torch.zeros(2, 256, device=DEV))


def test_config4_shape_properties():
    """Config 4 shape: Cl(7,1), x (2,097,152 x 256), beta ~ N(0, 0.1)."""
    batch = 2_097_152
    gen = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(batch, 256, device=DEV, generator=gen)
    beta = 0.1 * torch.randn(1, 28, device=DEV, generator=gen)
    cl = algebra(8, [1] * 7 + [-1])
    with torch.no_grad():
        y = cl.apply_bivector(beta, x)
    rows = torch.randperm(batch, generator=torch.Generator().manual_seed(0))[:64].to(DEV)
    ref = O.rotor_apply(8, beta.cpu().numpy().ravel(), x[rows].cpu().numpy())
    assert rel_l2(y[rows].cpu().numpy(), ref) <= REL_L2_TOL
    nx = torch.linalg.norm(x, dim=1)
    ny = torch.linalg.norm(y, dim=1)
    assert ((ny - nx).abs() / nx).max().item() < 1e-4
    _lib.device_status(DEV)


def test_rotor_unaligned_views():
    """x and the upstream gradient as views one float into their buffers:
    apply_bivector copies them to aligned rows; results match the aligned run."""
    n, batch = 8, 21
    cl = algebra(n)
    gen = torch.Generator(device=DEV).manual_seed(5)
    beta = (0.2 * torch.randn(1, 28, device=DEV, generator=gen)).requires_grad_(True)
    x = torch.randn(batch, 256, device=DEV, generator=gen)
    g = torch.randn(batch, 256, device=DEV, generator=gen)
    bx = torch.zeros(batch * 256 + 1, device=DEV)
    bx[1:].copy_(x.view(-1))
    bg = torch.zeros(batch * 256 + 1, device=DEV)
    bg[1:].copy_(g.view(-1))
    xv = bx[1:].view(batch, 256).requires_grad_(True)
    y = cl.apply_bivector(beta, xv)
    y.backward(bg[1:].view(batch, 256))
    x2 = x.clone().requires_grad_(True)
    beta2 = beta.detach().clone().requires_grad_(True)
    y2 = cl.apply_bivector(beta2, x2)
    y2.backward(g)
    assert rel_l2(y.detach().cpu().numpy(), y2.detach().cpu().numpy()) < 1e-6
    assert rel_l2(xv.grad.cpu().numpy(), x2.grad.cpu().numpy()) < 1e-6
    assert rel_l2(beta.grad.cpu().numpy(), beta2.grad.cpu().numpy()) < 1e-6
