"""Parity of the CUDA product path (through the C ABI) with the oracle.

* every product x the reference's signature spread, forward and both
  gradients, against the golden fixtures made from the reference;
* larger seeded batches at n = 5..10 (tiled and generic kernels) against the
  C oracle, including ragged batch sizes, an empty batch and unaligned
  pointers (which take the generic kernel);
* full-size properties at the BASELINE shapes: sampled rows against the
  oracle, and linearity in the second argument.
Tolerance: relative L2 <= 1e-5 against float64 (tests/helpers.py).
"""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib
from cliffordcuda_b200.products import bilinear_raw
from oracle import ga_oracle as O
from tests.helpers import (REL_L2_TOL, inputs, load_npz, product_cases, rel_l2,
                           signature_spread)

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

FUNCS = {"gp": cc.geom_prod, "wedge": cc.wedge_prod, "inner": cc.inner_prod,
         "lc": cc.left_contract, "rc": cc.right_contract, "reg": cc.regressive_prod}
OPS = ["gp", "wedge", "inner", "lc", "rc", "reg"]
CASES = product_cases()


def fwd_bwd_gpu(op, metric, a, b, g):
    at = torch.tensor(a, device=DEV, requires_grad=True)
    bt = torch.tensor(b, device=DEV, requires_grad=True)
    c = FUNCS[op](at, bt, metric=metric)
    c.backward(torch.tensor(g, device=DEV))
    return c.detach().cpu().numpy(), at.grad.cpu().numpy(), bt.grad.cpu().numpy()


@pytest.mark.parametrize("op,metric", CASES, ids=[f"{o}-{m}" for o, m in CASES])
def test_golden(op, metric):
    P = load_npz("products.npz")
    key = f"{op}|{','.join(map(str, metric))}"
    got = fwd_bwd_gpu(op, metric, P[key + "|a"], P[key + "|b"], P[key + "|g"])
    for mine, name in zip(got, ("c", "ga", "gb")):
        assert rel_l2(mine, P[key + "|" + name]) <= REL_L2_TOL, name


def test_config1():
    """Cl(5,0), batch 4096, upstream grad = ones."""
    G = load_npz("config1.npz")
    a, b, _ = inputs(5, int(G["seed"]), 4096)
    c, ga, gb = fwd_bwd_gpu("gp", (1,) * 5, a, b, np.ones_like(a))
    for arr, name, i in ((c, "c", 0), (ga, "ga", 1), (gb, "gb", 2)):
        assert rel_l2(arr[:64], G[name + "_head"]) <= REL_L2_TOL
        assert abs(np.linalg.norm(arr) - G["norms"][i]) <= 1e-5 * G["norms"][i]


def _check_all_modes(op, n, metric, batch, seed, offset=0):
    a, b, g = inputs(n, seed, batch)
    ref = O.forward_backward(op, n, metric, a, b, g)
    D = 1 << n
    tens = []
    for arr in (a, b, g):
        buf = torch.zeros(batch * D + offset, device=DEV)
        t = buf[offset:].view(batch, D)
        t.copy_(torch.from_numpy(arr))
        tens.append(t)
    ta, tb, tg = tens
    outs = []
    for mode, x, y in (("fwd", ta, tb), ("grad_a", tb, tg), ("grad_b", ta, tg)):
        obuf = torch.full((batch * D + offset,), float("nan"), device=DEV)
        o = obuf[offset:].view(batch, D)
        bilinear_raw(op, mode, x, y, n, metric, out=o)
        outs.append(o.cpu().numpy())
    for mine, r, name in zip(outs, ref, ("fwd", "grad_a", "grad_b")):
        err = rel_l2(mine, r)
        assert err <= REL_L2_TOL, f"{op} n={n} {metric} {name}: rel L2 {err:.3e}"


@pytest.mark.parametrize("n", [5, 6, 7, 8, 9, 10])
@pytest.mark.parametrize("op", OPS)
def test_tiled_sizes(op, n):
    # Euclidean low generators -> tiled kernel (reg -> generic); a negative
    # and (except reg) a null generator on top.
    top = [-1] if op == "reg" else [-1, 0]
    metric = tuple([1] * (n - len(top)) + top) if n > 5 else tuple([1] * n)
    batch = {5: 300, 6: 200, 7: 130, 8: 70, 9: 20, 10: 9}[n]
    _check_all_modes(op, n, metric, batch, seed=n * 10 + OPS.index(op))


@pytest.mark.parametrize("n", [5, 7, 9])
@pytest.mark.parametrize("sig", range(6))
def test_signature_spread(n, sig):
    metric = signature_spread(n)[sig]
    for op in OPS:
        if op == "reg" and 0 in metric:
            continue
        _check_all_modes(op, n, metric, 33, seed=100 + sig)


@pytest.mark.parametrize("batch", [1, 2, 3, 17, 255, 257])
def test_ragged_batches(batch):
    _check_all_modes("gp", 8, (1,) * 8, batch, seed=batch)
    _check_all_modes("inner", 7, (1,) * 6 + (-1,), batch, seed=batch + 1)


@pytest.mark.parametrize("op", ["gp", "inner", "lc"])
def test_unaligned_pointers_take_generic_path(op):
    _check_all_modes(op, 8, (1,) * 7 + (-1,), 19, seed=5, offset=1)


def test_empty_batch():
    a = torch.empty(0, 256, device=DEV)
    assert cc.geom_prod(a, a).shape == (0, 256)


def test_tiled_matches_generic():
    """Tiled (aligned) and generic (offset) paths agree to fp32 rounding."""
    n, batch = 8, 64
    a, b, _ = inputs(n, 9, batch)
    D = 1 << n
    ta = torch.tensor(a, device=DEV)
    tb = torch.tensor(b, device=DEV)
    t1 = bilinear_raw("gp", "fwd", ta, tb, n, (1,) * n)
    buf = torch.zeros(3, batch * D + 1, device=DEV)
    xa, xb, xo = (buf[i, 1:].view(batch, D) for i in range(3))
    xa.copy_(ta)
    xb.copy_(tb)
    bilinear_raw("gp", "fwd", xa, xb, n, (1,) * n, out=xo)
    assert rel_l2(t1.cpu().numpy(), xo.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("op,n,metric,batch", [
    ("gp", 8, (1,) * 8, 524288),                    # headline per-GPU shape
    ("gp", 7, (1,) * 6 + (-1,), 1 << 20),           # config 2
    ("wedge", 7, (1,) * 6 + (-1,), 1 << 20),
    ("inner", 7, (1,) * 6 + (-1,), 1 << 20),
    ("lc", 7, (1,) * 6 + (-1,), 1 << 20),
    ("rc", 7, (1,) * 6 + (-1,), 1 << 20),
    ("gp", 10, (1,) * 9 + (0,), 131072),            # config 5
    ("lc", 10, (1,) * 9 + (0,), 131072),
])
def test_full_size_properties(op, n, metric, batch):
    """At the BASELINE shapes: 64 sampled rows of each sum match the oracle,
    and the forward is linear in b (c(a, b1 + b2) = c(a, b1) + c(a, b2))."""
    D = 1 << n
    gen = torch.Generator(device=DEV).manual_seed(n)
    a = torch.randn(batch, D, device=DEV, generator=gen)
    b = torch.randn(batch, D, device=DEV, generator=gen)
    g = torch.randn(batch, D, device=DEV, generator=gen)
    rows = torch.randperm(batch, generator=torch.Generator().manual_seed(1))[:64].to(DEV)
    for mode, x, y in (("fwd", a, b), ("grad_a", b, g), ("grad_b", a, g)):
        out = bilinear_raw(op, mode, x, y, n, metric)
        ref = O.product(op, mode, n, metric, x[rows].cpu().numpy(), y[rows].cpu().numpy())
        assert rel_l2(out[rows].cpu().numpy(), ref) <= REL_L2_TOL, mode
        del out
    b2 = torch.randn(batch, D, device=DEV, generator=gen)
    lhs = bilinear_raw(op, "fwd", a, b + b2, n, metric)
    rhs = bilinear_raw(op, "fwd", a, b, n, metric) + bilinear_raw(op, "fwd", a, b2, n, metric)
    assert (torch.linalg.norm(lhs - rhs) / torch.linalg.norm(rhs)).item() < 1e-5
    _lib.device_status(DEV)


def test_algebra_methods_match_oracle():
    cl = cc.CliffordAlgebra([1, 1, 1, 1, 1, 1, -1], device=DEV)
    a, b, _ = inputs(7, 3, 5)
    ta, tb = torch.tensor(a, device=DEV), torch.tensor(b, device=DEV)
    pairs = [(cl.geom_prod, "gp"), (cl.wedge_prod, "wedge"), (cl.inner_prod, "inner"),
             (cl.left_contraction, "lc"), (cl.right_contraction, "rc"),
             (cl.regressive_prod, "reg")]
    for meth, op in pairs:
        got = meth(ta, tb).cpu().numpy()
        ref = O.forward_backward(op, 7, cl.metric, a, b, np.zeros_like(a))[0]
        assert rel_l2(got, ref) <= REL_L2_TOL, op


def test_device_status_clean():
    _lib.device_status(DEV)


@pytest.mark.parametrize("batch", [1, 7, 9, 257, 524288])
def test_fused_backward_cl8(batch):
    """cb_bilinear_bwd for the Cl(8,0) geometric product (both gradients from
    one pass over a, b, g; the matrix-representation kernel) against the
    oracle on ragged batches and, on sampled rows, at the headline shape;
    requesting one gradient takes the single-sum path and must agree."""
    from cliffordcuda_b200.products import bilinear_bwd_raw
    n, metric, D = 8, (1,) * 8, 256
    gen = torch.Generator(device=DEV).manual_seed(batch)
    a, b, g = (torch.randn(batch, D, device=DEV, generator=gen) for _ in range(3))
    ga, gb = torch.empty_like(a), torch.empty_like(a)
    bilinear_bwd_raw("gp", a, b, g, n, metric, ga, gb)
    rows = torch.arange(batch, device=DEV) if batch <= 512 else \
        torch.randperm(batch, generator=torch.Generator().manual_seed(2))[:64].to(DEV)
    _, ref_ga, ref_gb = O.forward_backward("gp", n, metric, a[rows].cpu().numpy(),
                                           b[rows].cpu().numpy(), g[rows].cpu().numpy())
    assert rel_l2(ga[rows].cpu().numpy(), ref_ga) <= REL_L2_TOL
    assert rel_l2(gb[rows].cpu().numpy(), ref_gb) <= REL_L2_TOL
    ga1, gb1 = torch.empty_like(a), torch.empty_like(a)
    bilinear_bwd_raw("gp", a, b, g, n, metric, ga1, None)
    bilinear_bwd_raw("gp", a, b, g, n, metric, None, gb1)
    assert rel_l2(ga1.cpu().numpy(), ga.cpu().numpy()) < 1e-6
    assert rel_l2(gb1.cpu().numpy(), gb.cpu().numpy()) < 1e-6
    _lib.device_status(DEV)


def test_fused_backward_rejects_aliasing():
    from cliffordcuda_b200.products import bilinear_bwd_raw
    a, b, g = (torch.randn(16, 256, device=DEV) for _ in range(3))
    with pytest.raises(_lib.CliffordNativeError):
        bilinear_bwd_raw("gp", a, b, g, 8, (1,) * 8, a, torch.empty_like(a))


def test_direct_path_cl8_gp():
    """cb_bilinear_direct keeps the blade-by-blade kernels for the Euclidean
    Cl(8,0) product: all three sums against the oracle, and against the
    matrix-representation route of cb_bilinear."""
    n, metric, batch = 8, (1,) * 8, 70
    a, b, g = inputs(n, 21, batch)
    ref = O.forward_backward("gp", n, metric, a, b, g)
    ta, tb, tg = (torch.tensor(v, device=DEV) for v in (a, b, g))
    for (mode, x, y), r in zip((("fwd", ta, tb), ("grad_a", tb, tg), ("grad_b", ta, tg)), ref):
        d = bilinear_raw("gp", mode, x, y, n, metric, direct=True)
        m = bilinear_raw("gp", mode, x, y, n, metric)
        assert rel_l2(d.cpu().numpy(), r) <= REL_L2_TOL, mode
        assert rel_l2(d.cpu().numpy(), m.cpu().numpy()) < 1e-6, mode


@pytest.mark.parametrize("metric", [
    (-1,) * 8,                                  # Cl(0,8): every low generator negative
    (1, 1, 1, 1, -1, -1, -1, -1),               # Cl(4,4): one negative low generator
    (1, -1, 1, -1, 1, -1, 1, -1, 1, -1),        # alternating: negatives relabelled
    (-1, 1, 1, -1, 1, 1, -1),                   # Cl(4,3), negatives at low bits 0 and 3
    (1, 1, -1, 1, 1, 0, -1, 1, 1),              # a null generator among the high bits
])
@pytest.mark.parametrize("op", ["gp", "wedge", "inner", "lc", "rc"])
def test_negative_low_generators_tiled(op, metric):
    """Metrics with generators squaring to -1 among the low five run the tiled
    kernel (the negatives relabelled to the top of the low block); aligned
    (tiled) against the oracle, and against the unaligned (generic) path."""
    n = len(metric)
    _check_all_modes(op, n, metric, 67, seed=n + len(op))
    _check_all_modes(op, n, metric, 19, seed=n + 1, offset=1)


@pytest.mark.parametrize("batch", [1, 5, 333])
def test_pga10_route(batch):
    """The Cl(9,0,1) geometric product goes through six Cl(8,0) matrix
    products per sum (cb_bilinear_ws / cb_bilinear_bwd_ws); against the oracle,
    and against the blade-by-blade kernels (cb_bilinear_direct)."""
    n, metric = 10, (1,) * 9 + (0,)
    a, b, g = inputs(n, 40 + batch, batch)
    ref = O.forward_backward("gp", n, metric, a, b, g)
    got = fwd_bwd_gpu("gp", metric, a, b, g)
    for mine, r, name in zip(got, ref, ("c", "ga", "gb")):
        assert rel_l2(mine, r) <= REL_L2_TOL, name
    ta, tb = torch.tensor(a, device=DEV), torch.tensor(b, device=DEV)
    d = bilinear_raw("gp", "fwd", ta, tb, n, metric, direct=True)
    assert rel_l2(got[0], d.cpu().numpy()) < 1e-6


@pytest.mark.parametrize("op", ["wedge", "lc", "rc", "reg", "inner"])
@pytest.mark.parametrize("n,top", [(9, (0,)), (10, (0, 0)), (10, (-1,)), (8, (0, -1))])
def test_balanced_step_schedule(op, n, top):
    """The sparse products at n = 8..10 run under the balanced step schedule
    (heavy output blocks lend step segments to light lanes; the lent sums come
    back through the row's y lines), the inner product under its two-phase
    form (LC rounds, then RC rounds): null high generators change the per-block
    step counts, and every mode has its own pattern."""
    if op == "reg" and 0 in top:
        top = tuple(-1 if v == 0 else v for v in top)
    metric = tuple([1] * (n - len(top)) + list(top))
    _check_all_modes(op, n, metric, 13, seed=7 * n + len(top))


@pytest.mark.parametrize("batch", [1, 31, 33, 4096])
def test_cl61_route(batch):
    """Cl(6,1) geometric product through two Cl(6,0) sums per row (the tiled
    kernel's pseudoscalar route): all three sums against the oracle, ragged
    tiles included, and the route agrees with the blade-by-blade kernel."""
    metric = (1,) * 6 + (-1,)
    _check_all_modes("gp", 7, metric, batch, seed=61 + batch)
    a, b, _ = inputs(7, 5, batch)
    ta, tb = torch.tensor(a, device=DEV), torch.tensor(b, device=DEV)
    rep = bilinear_raw("gp", "fwd", ta, tb, 7, metric)
    buf = torch.zeros(3, batch * 128 + 1, device=DEV)      # offset views: generic kernel
    xa, xb, xo = (buf[i, 1:].view(batch, 128) for i in range(3))
    xa.copy_(ta)
    xb.copy_(tb)
    bilinear_raw("gp", "fwd", xa, xb, 7, metric, out=xo)
    assert rel_l2(rep.cpu().numpy(), xo.cpu().numpy()) < 1e-6
