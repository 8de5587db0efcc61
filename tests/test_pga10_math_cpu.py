"""The algebra behind the Cl(9,0,1) route (csrc/pga10.cu, gp9_kernel), checked in
float64 with the oracle's Cl(8,0) and Cl(9,0,1) sums, no GPU:

* dual numbers: a = a0 + a1 e9 gives c0 = a0 b0, c1 = a0 b1 + a1 g(b0);
* Cl(9,0) = Cl(8,0) + Cl(8,0): x = u + v e8 -> (u + v w, u - v w), w = e0...e7,
  back by u = (P + Q)/2, v = (P - Q) w / 2 (also the adjoint the backward uses);
* the backward sums through the same maps:
  grad_a0 = gA(b0; g0) + gA(b1; g1), grad_a1 = gA(g(b0); g1),
  grad_b0 = gB(a0; g0) + g(gB(a1; g1)), grad_b1 = gB(a0; g1);
* g(gB(a1; g1)) = gB(g(a1); g(g1)) (g an orthogonal automorphism), the form the
  kernel sums in the matrix domain.
"""
import numpy as np

from oracle import ga_oracle as O

E8, M10 = (1,) * 8, (1,) * 9 + (0,)
IDX = np.arange(256)
W = np.where(np.array([sum(t for t in range(8) if (k >> t) & 1) for k in range(256)]) % 2, -1.0, 1.0)
G8 = np.where(np.array([bin(k).count("1") % 2 for k in range(256)]) == 1, -1.0, 1.0)


def omega(v):            # (v w)[K] = w(~K) v[~K]
    return v[:, 255 - IDX] * W[255 - IDX]


def split(x):            # Cl(9,0) block -> its two Cl(8,0) components
    u, v = x[:, :256], x[:, 256:]
    return u + omega(v), u - omega(v)


def merge(P, Q):         # the inverse map (1/2 of the adjoint)
    return np.concatenate([P + Q, omega(P - Q)], 1) / 2


def ginv9(x):            # grade involution of a Cl(9,0) block: g(u) - g(v) e8
    return np.concatenate([x[:, :256] * G8, -x[:, 256:] * G8], 1)


def s9(mode, x, y):      # one Cl(9,0) sum through the components
    xp, xm = split(x)
    yp, ym = split(y)
    return merge(O.product("gp", mode, 8, E8, xp, yp), O.product("gp", mode, 8, E8, xm, ym))


def test_cl901_product_and_gradients_through_cl8():
    rng = np.random.default_rng(0)
    a, b, g = (rng.standard_normal((3, 1024)) for _ in range(3))
    a0, a1, b0, b1, g0, g1 = a[:, :512], a[:, 512:], b[:, :512], b[:, 512:], g[:, :512], g[:, 512:]
    c = np.concatenate([s9("fwd", a0, b0), s9("fwd", a0, b1) + s9("fwd", a1, ginv9(b0))], 1)
    ga = np.concatenate([s9("grad_a", b0, g0) + s9("grad_a", b1, g1),
                         s9("grad_a", ginv9(b0), g1)], 1)
    gb = np.concatenate([s9("grad_b", a0, g0) + ginv9(s9("grad_b", a1, g1)),
                         s9("grad_b", a0, g1)], 1)
    ref = O.forward_backward("gp", 10, M10, a, b, g)
    for mine, r in zip((c, ga, gb), ref):
        assert np.abs(mine - r).max() <= 1e-12 * np.abs(r).max()
    alt = s9("grad_b", ginv9(a1), ginv9(g1))
    ref_t = ginv9(s9("grad_b", a1, g1))
    assert np.abs(alt - ref_t).max() <= 1e-12 * np.abs(ref_t).max()
