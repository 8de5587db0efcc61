"""The large-n regime (n = 11..16): the reference hands these to its tiled
fused product (extensions/ga/geom_prod_tiled.py:370-398); here the wide
kernel (csrc/bilinear_wide.cuh) for metrics whose low five generators square
to +1, the generic kernels otherwise (and for the regressive product).

* the golden fixtures computed with the reference's einsum at n = 11..14
  (tests/golden/large_n.npz), through the public API with autograd;
* every product at n = 11 and 12 over signatures that take each kernel;
* n = 15 and 16 with the reference's own past-the-limit signatures
  (tests/correctness/test_geom_prod_tiled.py:134-138) against the C oracle;
* batch shapes that split output blocks over CTAs (one row) and that do not
  (many rows, sampled), ragged two-row blocks at n = 11, unaligned views.
Tolerance: relative L2 <= 1e-5 against float64 (tests/helpers.py).
"""
import numpy as np
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib
from cliffordcuda_b200.products import bilinear_raw
from oracle import ga_oracle as O
from tests.helpers import REL_L2_TOL, inputs, load_npz, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
FUNCS = {"gp": cc.geom_prod, "wedge": cc.wedge_prod, "inner": cc.inner_prod,
         "lc": cc.left_contract, "rc": cc.right_contract, "reg": cc.regressive_prod}


def _cases():
    P = load_npz("large_n.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in P.files})
    return [(k.split("|")[0], tuple(int(v) for v in k.split("|")[1].split(","))) for k in keys]


def _fwd_bwd(op, metric, a, b, g):
    at = torch.tensor(a, device=DEV, requires_grad=True)
    bt = torch.tensor(b, device=DEV, requires_grad=True)
    c = FUNCS[op](at, bt, metric=metric)
    c.backward(torch.tensor(g, device=DEV))
    return c.detach().cpu().numpy(), at.grad.cpu().numpy(), bt.grad.cpu().numpy()


@pytest.mark.parametrize("op,metric", _cases(),
                         ids=[f"{o}-n{len(m)}-{i}" for i, (o, m) in enumerate(_cases())])
def test_golden_large_n(op, metric):
    P = load_npz("large_n.npz")
    key = f"{op}|{','.join(map(str, metric))}"
    got = _fwd_bwd(op, metric, P[key + "|a"], P[key + "|b"], P[key + "|g"])
    for mine, name in zip(got, ("c", "ga", "gb")):
        err = rel_l2(mine, P[key + "|" + name])
        assert err <= REL_L2_TOL, f"{key} {name}: rel L2 {err:.3e}"
    _lib.device_status(DEV)


def _check(op, n, metric, batch, seed, rows=None, offset=0):
    a, b, g = inputs(n, seed, batch)
    D = 1 << n
    tens = []
    for arr in (a, b, g):
        buf = torch.zeros(batch * D + offset, device=DEV)
        t = buf[offset:].view(batch, D)
        t.copy_(torch.from_numpy(arr))
        tens.append(t)
    ta, tb, tg = tens
    sel = np.arange(batch) if rows is None else rows
    for mode, x, y, xn, yn in (("fwd", ta, tb, a, b), ("grad_a", tb, tg, b, g),
                               ("grad_b", ta, tg, a, g)):
        out = bilinear_raw(op, mode, x, y, n, metric)
        if op == "reg":
            ref = O.forward_backward("reg", n, metric, a[sel], b[sel], g[sel])
            ref = ref[{"fwd": 0, "grad_a": 1, "grad_b": 2}[mode]]
        else:
            ref = O.product(op, mode, n, metric, xn[sel], yn[sel])
        err = rel_l2(out.cpu().numpy()[sel], ref)
        assert err <= REL_L2_TOL, f"{op} n={n} {metric} {mode}: rel L2 {err:.3e}"


@pytest.mark.parametrize("n", [11, 12])
@pytest.mark.parametrize("op", ["gp", "wedge", "inner", "lc", "rc", "reg"])
@pytest.mark.parametrize("sig", ["euclid_low", "mixed_low"])
def test_products_n11_n12(op, n, sig):
    if sig == "euclid_low":   # wide kernel (generic for reg)
        metric = (1,) * (n - 3) + ((-1, -1, -1) if op == "reg" else (-1, 0, -1))
    else:                     # generic kernels
        metric = tuple((1, -1, 1, -1)[i % 4] for i in range(n))
    _check(op, n, metric, 3, seed=100 * n + len(op))


@pytest.mark.parametrize("n,metric,batch", [
    (13, (1,) * 13, 1),
    (14, (1,) * 12 + (-1, -1), 1),
    (15, (1,) * 9 + (-1,) * 6, 2),
    (16, (1,) * 13 + (-1, -1, 0), 1),
])
def test_gp_past_the_limit(n, metric, batch):
    _check("gp", n, metric, batch, seed=n)


@pytest.mark.parametrize("op", ["inner", "lc", "wedge"])
def test_products_n14(op):
    _check(op, 14, (1,) * 11 + (-1, -1, 0), 1, seed=14 + len(op))


def test_generic_large_rows():
    """Non-Euclidean low generators and the regressive product at n = 13, 14
    take the unstaged generic kernel."""
    _check("gp", 13, tuple((1, 1, 1, -1, -1, 0)[i % 6] for i in range(13)), 1, seed=3)
    _check("reg", 13, (1,) * 11 + (-1, -1), 1, seed=4)
    _check("lc", 14, (-1,) * 14, 1, seed=5)


@pytest.mark.parametrize("n,batch", [(11, 1), (11, 3), (11, 2001), (12, 600), (13, 150)])
def test_batches_and_splits(n, batch):
    """One row (output blocks split over CTAs, atomics), an odd number of rows
    at n = 11 (two-row blocks with a zero-filled tail), and enough rows that
    nothing is split (sampled rows against the oracle)."""
    metric = (1,) * (n - 1) + (-1,)
    rows = None if batch <= 3 else np.random.default_rng(batch).choice(batch, 4, replace=False)
    _check("gp", n, metric, batch, seed=batch, rows=rows)
    _check("inner", n, metric, batch, seed=batch + 1, rows=rows)
    _lib.device_status(DEV)


def test_unaligned_large_n():
    _check("gp", 12, (1,) * 11 + (-1,), 2, seed=9, offset=1)
    _check("lc", 13, (1,) * 13, 1, seed=10, offset=3)
