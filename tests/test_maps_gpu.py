"""The per-blade maps and norm_sq on the native kernels (cb_blade_map,
cb_norm_sq) against the reference's own outputs (tests/golden/maps.npz,
made by tests/golden/make_golden_maps.py) and the oracle.

Sign maps multiply by +-1 / 0, so they are bit-exact; norm_sq sums in a
different order than torch and is held to relative 1e-6. Gradients are the
transposed maps, checked against float64 autograd of the oracle's matrices.
"""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib, blade_maps
from oracle import ga_oracle as O
from tests.helpers import load_npz, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _keys():
    return sorted({k.split("|")[0] for k in load_npz("maps.npz").files})


@pytest.mark.parametrize("key", _keys())
def test_maps_match_reference_outputs(key):
    M = load_npz("maps.npz")
    metric = [int(v) for v in key.split(",")]
    n = len(metric)
    cl = cc.CliffordAlgebra(metric, device=DEV)
    x = torch.tensor(M[key + "|x"], device=DEV)
    got = {"reverse": cl.reverse(x), "involute": cl.grade_involution(x),
           "conjugate": cl.clifford_conjugation(x), "free_reverse": cc.reverse(x)}
    for name, t in got.items():
        assert np.array_equal(t.cpu().numpy(), M[key + "|" + name]), name
    for k in range(n + 1):
        assert np.array_equal(cl.grade_projection(x, k).cpu().numpy(), M[key + "|grade"][k])
    if 0 not in metric:
        assert np.array_equal(cl.dual(x).cpu().numpy(), M[key + "|dual"])
    else:
        with pytest.raises(ValueError):
            cl.dual(x)
    ns = cl.norm_sq(x).cpu().numpy()
    ref = M[key + "|norm_sq"].astype(np.float64)
    assert np.allclose(ns, ref, rtol=1e-6, atol=1e-6 * np.abs(ref).max())


@pytest.mark.parametrize("n,metric", [(1, (1,)), (2, (-1, 1)), (3, (1, 0, -1)),
                                      (8, (1,) * 7 + (-1,)), (10, (1,) * 9 + (0,)),
                                      (12, (1,) * 10 + (-1, 1))])
@pytest.mark.parametrize("batch", [1, 7, 1000])
def test_maps_sizes_and_gradients(n, metric, batch):
    """Every map at small and large n (scalar and float4 paths), forward
    against the oracle (bit-exact) and backward against the transposed map."""
    rng = np.random.default_rng(n * 100 + batch)
    D = 1 << n
    x = rng.standard_normal((batch, D)).astype(np.float32)
    g = rng.standard_normal((batch, D)).astype(np.float32)
    kinds = ["reverse", "involute", "conjugate", "grade"] + ([] if 0 in metric else ["dual"])
    for kind in kinds:
        grade = n // 2
        xt = torch.tensor(x, device=DEV, requires_grad=True)
        y = blade_maps.blade_map(kind, xt, metric, grade)
        y.backward(torch.tensor(g, device=DEV))
        ref = O.blade_map(kind, n, metric, x, grade)
        assert np.array_equal(y.detach().cpu().numpy(), ref.astype(np.float32)), kind
        tkind = "dual_t" if kind == "dual" else kind
        assert np.array_equal(xt.grad.cpu().numpy(),
                              O.blade_map(tkind, n, metric, g, grade).astype(np.float32)), kind
    xt = torch.tensor(x, device=DEV, requires_grad=True)
    s = blade_maps.norm_sq(xt, metric)
    gs = rng.standard_normal(batch).astype(np.float32)
    s.backward(torch.tensor(gs, device=DEV))
    ref = O.norm_sq(n, metric, x)
    assert rel_l2(s.detach().cpu().numpy(), ref) < 1e-6
    w = O.norm_sq(n, metric, np.eye(D))              # the per-blade weights
    assert rel_l2(xt.grad.cpu().numpy(), 2 * w * x * gs[:, None]) < 1e-6
    _lib.device_status(DEV)


def test_maps_unaligned_and_empty():
    """Views one float into their buffer take the scalar path; same results."""
    n, metric, batch = 7, (1,) * 6 + (-1,), 33
    rng = np.random.default_rng(3)
    x = rng.standard_normal((batch, 128)).astype(np.float32)
    buf = torch.zeros(batch * 128 + 1, device=DEV)
    buf[1:].copy_(torch.from_numpy(x).view(-1))
    xv = buf[1:].view(batch, 128)
    for kind in ("reverse", "dual", "grade"):
        out = blade_maps.map_raw(kind, xv, n, metric, 3)
        assert np.array_equal(out.cpu().numpy(),
                              O.blade_map(kind, n, metric, x, 3).astype(np.float32)), kind
    empty = torch.empty(0, 128, device=DEV)
    assert blade_maps.map_raw("reverse", empty, n, metric).shape == (0, 128)
    assert blade_maps.norm_sq(empty, metric).shape == (0,)


def test_maps_large_batch_bandwidth_shape():
    """At a config-2-sized batch (1,048,576 x 128) the float4 path matches the
    oracle on sampled rows and the dual is an involution up to I^2 signs:
    dual_t(dual(x)) = x."""
    n, metric, batch = 7, (1,) * 6 + (-1,), 1 << 20
    gen = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(batch, 128, device=DEV, generator=gen)
    y = blade_maps.map_raw("dual", x, n, metric)
    back = blade_maps.map_raw("dual_t", y, n, metric)
    assert torch.equal(back, x)
    rows = torch.randperm(batch, generator=torch.Generator().manual_seed(1))[:64].to(DEV)
    ref = O.blade_map("dual", n, metric, x[rows].cpu().numpy())
    assert np.array_equal(y[rows].cpu().numpy(), ref.astype(np.float32))
    _lib.device_status(DEV)
