"""The real 16 x 16 matrix representation behind the Cl(8,0) matrix route
(cliffordcuda_b200/csrc/mat16_rep.cuh), checked on the CPU:

* the constexpr tables of the header, compiled on the host with g++, rebuild
  generator matrices that square to 1 and anticommute;
* a numpy model of the kernels' per-lane algorithm (gather with the slot and
  sign tables, in-register butterflies, the factor-4 shuffle stage, the
  quadrant layout and the inverse) reproduces the oracle's geometric product
  and both of its backward sums, for the forward and the two transposed
  forms the backward kernels use.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import ga_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "cliffordcuda_b200", "csrc", "mat16_rep.cuh")

PROG = r"""
#include <cstdio>
#define __host__
#define __device__
#include "HDR"
using namespace cb::mat16;
int main() {
    for (int i = 0; i < 6; ++i) for (int f = 0; f < 3; ++f) printf("%d ", kP(i, f));
    printf("\n");
    for (int k = 0; k < 64; ++k) printf("%d ", slot_of(k));
    printf("\n");
    for (int k = 0; k < 64; ++k) printf("%d ", sig1_of(k));
    printf("\n");
    for (int q = 0; q < 4; ++q) for (int m = 0; m < 4; ++m) printf("%d ", last_sign(q, m));
    printf("\n");
    for (int i = 0; i < 8; ++i) for (int j = 0; j < 8; ++j) printf("%d ", slot_ij(i, j));
    printf("\n");
}
"""

P2 = {0: np.eye(2), 1: np.array([[0., 1], [1, 0]]), 2: np.array([[1., 0], [0, -1]]),
      3: np.array([[0., -1], [1, 0]])}


@pytest.fixture(scope="module")
def tables(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    d = tmp_path_factory.mktemp("mat16")
    src = d / "t.cpp"
    src.write_text(PROG.replace("HDR", HDR))
    exe = d / "t"
    subprocess.run(["g++", "-std=c++17", "-O1", str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], check=True, capture_output=True,
                           text=True).stdout.splitlines()
    nums = [[int(v) for v in ln.split()] for ln in lines]
    return {"kP": np.array(nums[0]).reshape(6, 3), "slot": nums[1], "sig1": nums[2],
            "last": np.array(nums[3]).reshape(4, 4), "slot_ij": np.array(nums[4]).reshape(8, 8)}


def kron(codes):
    m = np.eye(1)
    for c in codes:
        m = np.kron(m, P2[c])
    return m


def gammas(kP):
    return [kron((0, 0, 0, 1)), kron((0, 0, 0, 2))] + [kron(tuple(p) + (3,)) for p in kP]


def test_generators(tables):
    G = gammas(tables["kP"])
    for i in range(8):
        assert np.array_equal(G[i], G[i].T)
        assert np.allclose(G[i] @ G[i], np.eye(16))
        for j in range(i):
            assert np.allclose(G[i] @ G[j], -G[j] @ G[i])
    assert sorted(tables["slot"]) == list(range(64))


class LaneModel:
    """The kernels' per-lane arithmetic, lane q of a product holding 64 slots."""

    def __init__(self, t):
        self.t = t
        lam = [1, 1, -1, 1]
        self.s_in = [[t["last"][q][m] * lam[q] for m in range(4)] for q in range(4)]
        self.s_out = [[t["last"][q][m] * lam[q] / 16 for m in range(4)] for q in range(4)]

    @staticmethod
    def blade(k, q):
        return 4 * k + (q ^ (3 if bin(k).count("1") & 1 else 0))

    def to_quadrants(self, x):
        t, r = self.t, np.zeros((4, 64))
        for q in range(4):
            for k in range(64):
                m = bin(k).count("1") & 3
                r[q, t["slot"][k]] = t["sig1"][k] * self.s_in[q][m] * x[self.blade(k, q)]
        for q in range(4):
            for f in range(3):
                tb, sb = 5 - 2 * f, 4 - 2 * f
                old = r[q].copy()
                for s in range(64):
                    if s >> tb & 1:
                        continue
                    p0, p1 = old[s], old[s | 1 << tb]
                    hi, lo = (p0 - p1, p0 + p1) if s >> sb & 1 else (p0 + p1, p0 - p1)
                    r[q, s], r[q, s | 1 << tb] = hi, lo
        c_fwd = [-1, -1, 1, 1]
        return np.array([r[q] + c_fwd[q] * r[q ^ 2] for q in range(4)])

    def matrix(self, r):
        M = np.zeros((16, 16))
        for q in range(4):
            r4, c4 = q >> 1, (q >> 1) ^ (q & 1)
            for i in range(8):
                for j in range(8):
                    M[2 * i + r4, 2 * j + c4] = r[q, self.t["slot_ij"][i, j]]
        return M

    def quadrants(self, M):
        r = np.zeros((4, 64))
        for q in range(4):
            r4, c4 = q >> 1, (q >> 1) ^ (q & 1)
            for i in range(8):
                for j in range(8):
                    r[q, self.t["slot_ij"][i, j]] = M[2 * i + r4, 2 * j + c4]
        return r

    def to_blades(self, r):
        t = self.t
        c_inv = [1, 1, -1, -1]
        r = np.array([r[q] + c_inv[q] * r[q ^ 2] for q in range(4)])
        for q in range(4):
            for f in range(3):
                tb, sb = 5 - 2 * f, 4 - 2 * f
                old = r[q].copy()
                for s in range(64):
                    if s >> tb & 1:
                        continue
                    m0, m1 = old[s], old[s | 1 << tb]
                    r[q, s] = m0 + m1
                    r[q, s | 1 << tb] = m1 - m0 if s >> sb & 1 else m0 - m1
        x = np.zeros(256)
        for q in range(4):
            for k in range(64):
                m = bin(k).count("1") & 3
                x[self.blade(k, q)] = t["sig1"][k] * self.s_out[q][m] * r[q, t["slot"][k]]
        return x


def test_lane_model_matches_oracle(tables):
    L = LaneModel(tables)
    rng = np.random.default_rng(7)
    a, b, g = rng.standard_normal((3, 2, 256))
    y, ga, gb = O.forward_backward("gp", 8, (1,) * 8, a, b, g)
    for row in range(2):
        A = L.matrix(L.to_quadrants(a[row]))
        B = L.matrix(L.to_quadrants(b[row]))
        Gm = L.matrix(L.to_quadrants(g[row]))
        for M, ref in ((A @ B, y), (Gm @ B.T, ga), (A.T @ Gm, gb)):
            got = L.to_blades(L.quadrants(M))
            assert np.abs(got - ref[row]).max() < 1e-12
