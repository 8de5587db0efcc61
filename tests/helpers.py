"""Shared test helpers: seeded inputs, golden fixtures, tolerance checks."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Acceptance: the fp32 CUDA path against float64 truth, relative L2. The
# north-star bar is 1e-4 against fp64 and 1e-5 against the reference's fp32
# result; fp32 rounding of these sums sits near 1e-7, so 1e-5 against fp64
# implies both.
REL_L2_TOL = 1e-5


def rel_l2(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(got - ref)
    return num / den if den > 0 else num


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name))


def product_cases():
    P = load_npz("products.npz")
    keys = sorted({k.rsplit("|", 1)[0] for k in P.files})
    out = []
    for k in keys:
        op, m = k.split("|")
        out.append((op, tuple(int(x) for x in m.split(","))))
    return out


def inputs(n, seed, batch, count=3):
    rng = np.random.default_rng(seed)
    D = 1 << n
    return [rng.standard_normal((batch, D)).astype(np.float32) for _ in range(count)]


def signature_spread(n):
    """The reference's six signatures per n (tests/_gradcheck.py:9-19)."""
    return [tuple([1] * n), tuple([-1] * n), tuple([1] * (n - 1) + [-1]),
            tuple([1] * (n // 2) + [-1] * (n - n // 2)),
            tuple([1] * (n - 1) + [0]), tuple([1] * (n - 2) + [-1, 0])]
