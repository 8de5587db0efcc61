"""The CPU oracle against the golden fixtures generated from the reference
(tests/golden/make_golden.py). No GPU."""
import hashlib

import numpy as np
import pytest

from oracle import ga_oracle as O
from tests.helpers import inputs, load_npz, product_cases, rel_l2

CASES = product_cases()


@pytest.mark.parametrize("op,metric", CASES, ids=[f"{o}-{m}" for o, m in CASES])
def test_products_vs_reference(op, metric):
    P = load_npz("products.npz")
    key = f"{op}|{','.join(map(str, metric))}"
    n = len(metric)
    c, ga, gb = O.forward_backward(op, n, metric, P[key + "|a"], P[key + "|b"], P[key + "|g"])
    for mine, name in ((c, "c"), (ga, "ga"), (gb, "gb")):
        ref = P[key + "|" + name]
        assert np.abs(mine - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max()), name


def test_config1_vs_reference():
    G = load_npz("config1.npz")
    a, b, _ = inputs(5, int(G["seed"]), 4096)
    g = np.ones_like(a)
    c, ga, gb = O.forward_backward("gp", 5, (1,) * 5, a, b, g)
    for arr, name, i in ((c, "c", 0), (ga, "ga", 1), (gb, "gb", 2)):
        np.testing.assert_allclose(arr[:64], G[name + "_head"], rtol=0, atol=1e-12)
        assert abs(arr.sum() - G["sums"][i]) <= 1e-9 * max(1, abs(G["sums"][i]))
        assert abs(np.linalg.norm(arr) - G["norms"][i]) <= 1e-9 * G["norms"][i]


def test_sign_tables_vs_reference():
    S = load_npz("sigma.npz")
    for key in S.files:
        kind, m = key.split("|")
        if kind != "gp":
            continue
        metric = tuple(int(x) for x in m.split(","))
        t = O.sign_table(len(metric), metric)
        assert hashlib.sha256(t.tobytes()).digest() == S[key].tobytes(), key


@pytest.mark.parametrize("n", [7, 8])
def test_rotor_vs_reference(n):
    R = load_npz("rotor.npz")
    beta, x, y = R[f"{n}|beta"], R[f"{n}|x"], R[f"{n}|y"]
    assert rel_l2(O.rotor_apply(n, beta, x), y) < 1e-12
    # the blade-minor form equals the reference's Givens chain
    chain = O.givens_chain_apply(n, O.rotor_matrix(n, beta), x)
    assert rel_l2(chain, y) < 1e-12


def test_rotor_matrix_orthogonal():
    rng = np.random.default_rng(3)
    Rm = O.rotor_matrix(8, rng.standard_normal(28))
    np.testing.assert_allclose(Rm @ Rm.T, np.eye(8), atol=1e-12)
    assert abs(np.linalg.det(Rm) - 1) < 1e-12


def test_einsum_port_matches_c_oracle():
    import torch
    a, b = [np.random.default_rng(5 + i).standard_normal((4, 64)) for i in range(2)]
    for op in ("gp", "wedge", "inner", "lc", "rc", "reg"):
        metric = (1, 1, 1, -1, 1, -1)
        f = O.EinsumProduct(op, 6, metric, dtype=torch.float64)
        got = f(torch.tensor(a), torch.tensor(b)).numpy()
        ref = O.regressive_fwd(6, metric, a, b) if op == "reg" else O.product(op, "fwd", 6, metric, a, b)
        assert rel_l2(got, ref) < 1e-13, op


def test_rotor_gradient_truth_matches_finite_differences():
    """The fp64 autograd truth used for the rotor gradients agrees with central
    differences of the oracle's forward map."""
    rng = np.random.default_rng(11)
    n = 7
    beta = 0.2 * rng.standard_normal(21)
    x, g = rng.standard_normal((2, 3, 128))
    y, dx, db = O.rotor_grads_torch(n, beta, x, g)
    eps = 1e-6
    for i in (0, 7, 20):
        bp, bm = beta.copy(), beta.copy()
        bp[i] += eps
        bm[i] -= eps
        fd = ((O.rotor_apply(n, bp, x) - O.rotor_apply(n, bm, x)) * g).sum() / (2 * eps)
        assert abs(fd - db[i]) <= 1e-6 * max(1.0, abs(db[i]))
    np.testing.assert_allclose(dx, g @ O.rotor_blade_matrix(n, O.rotor_matrix(n, beta)).T,
                               atol=1e-12)


@pytest.mark.parametrize("op", ["gp", "wedge", "inner", "lc", "rc"])
def test_layer_dw_from_G_matches_summed_grad_b(op):
    """The batch-free weight-gradient check used at full layer shapes equals
    the expand_as formulation: grad_b(x, w repeated; dy) summed over rows."""
    n, metric = 6, (1, 1, 1, -1, 1, 0)
    rng = np.random.default_rng(3)
    x, dy = (rng.standard_normal((40, 64)) for _ in range(2))
    w = rng.standard_normal(64)
    wrep = np.repeat(w.reshape(1, -1), 40, axis=0)
    dw_ref = O.forward_backward(op, n, metric, x, wrep, dy)[2].sum(axis=0)
    dw = O.layer_dw_from_G(op, n, metric, x.T @ dy)
    assert np.max(np.abs(dw - dw_ref)) < 1e-9 * np.max(np.abs(dw_ref))


def test_rotor_dbeta_from_G_matches_autograd():
    n = 7
    rng = np.random.default_rng(8)
    beta = 0.3 * rng.standard_normal(21)
    x, g = (rng.standard_normal((12, 128)) for _ in range(2))
    db_ref = O.rotor_grads_torch(n, beta, x, g)[2]
    db = O.rotor_dbeta_from_G(n, beta, x.T @ g)
    assert np.max(np.abs(db - db_ref)) < 1e-10 * np.max(np.abs(db_ref))


def _map_cases():
    M = load_npz("maps.npz")
    return sorted({k.split("|")[0] for k in M.files})


@pytest.mark.parametrize("key", _map_cases())
def test_blade_maps_vs_reference(key):
    M = load_npz("maps.npz")
    metric = tuple(int(v) for v in key.split(","))
    n = len(metric)
    x = M[key + "|x"]
    for kind in ("reverse", "involute", "conjugate"):
        assert np.array_equal(O.blade_map(kind, n, metric, x), M[key + "|" + kind]), kind
    assert np.array_equal(O.blade_map("reverse", n, metric, x), M[key + "|free_reverse"])
    for g in range(n + 1):
        assert np.array_equal(O.blade_map("grade", n, metric, x, g), M[key + "|grade"][g])
    if 0 not in metric:
        assert np.array_equal(O.blade_map("dual", n, metric, x), M[key + "|dual"])
        # dual_t is the transpose: <dual(x), y> = <x, dual_t(y)>
        y = np.random.default_rng(1).standard_normal(x.shape)
        lhs = (O.blade_map("dual", n, metric, x) * y).sum()
        rhs = (x * O.blade_map("dual_t", n, metric, y)).sum()
        assert abs(lhs - rhs) < 1e-10 * max(1.0, abs(lhs))
    ref = M[key + "|norm_sq"].astype(np.float64)
    assert np.allclose(O.norm_sq(n, metric, x), ref, rtol=1e-5, atol=1e-5)


def _large_cases():
    P = load_npz("large_n.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in P.files})
    return [(k.split("|")[0], tuple(int(v) for v in k.split("|")[1].split(","))) for k in keys]


@pytest.mark.parametrize("op,metric", _large_cases(),
                         ids=[f"{o}-n{len(m)}-{i}" for i, (o, m) in enumerate(_large_cases())])
def test_large_n_vs_reference(op, metric):
    """n = 11..14: the oracle against the reference's einsum (large_n.npz)."""
    P = load_npz("large_n.npz")
    key = f"{op}|{','.join(map(str, metric))}"
    n = len(metric)
    c, ga, gb = O.forward_backward(op, n, metric, P[key + "|a"], P[key + "|b"], P[key + "|g"])
    for mine, name in ((c, "c"), (ga, "ga"), (gb, "gb")):
        ref = P[key + "|" + name]
        assert np.abs(mine - ref).max() <= 1e-10 * max(1.0, np.abs(ref).max()), name


@pytest.mark.parametrize("op", ["gp", "wedge", "inner", "lc", "rc"])
def test_table_free_product_matches_table(op):
    """The table-free per-term sign used for n >= 11 equals the table path."""
    n, metric = 7, (1, -1, 0, 1, 1, -1, 1)
    rng = np.random.default_rng(2)
    x, y = (rng.standard_normal((3, 128)) for _ in range(2))
    m = O._metric_arr(metric)
    for mode in ("fwd", "grad_a", "grad_b"):
        ref = O.product(op, mode, n, metric, x, y)
        out = np.empty_like(ref)
        O.lib().orc_product_range(O.OPS[op], O.MODES[mode], n, m, 3, O._dptr(x), O._dptr(y),
                                  O._dptr(out), 0, 128)
        assert np.array_equal(out, ref), mode
