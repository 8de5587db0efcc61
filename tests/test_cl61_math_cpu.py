"""The algebra behind the Cl(6,1) route of the tiled kernel (bilinear_tiled.cuh,
PHI61), checked in float64 against the oracle's blade sums, no GPU.

With omega = e0 e1 ... e6 (central, omega^2 = +1 in Cl(6,1)) every x is
u + v omega with u, v even, and x -> (u + v, u - v) is an algebra isomorphism
onto pairs of elements of the even subalgebra, multiplied componentwise. The
even subalgebra is Cl(6,0) through f_i = e_i e_6. In coordinates: for each
Cl(6,0) blade k, f_k = a(k) e_E(k) and e_O omega = s(O) e_(O ^ 127), so
    P[k] = a(k) x[E] + b(k) x[O],  Q[k] = a(k) x[E] - b(k) x[O],
    E = E(k), O = E ^ 127, b(k) = a(k) s(O);
back, x[E] = a (P + Q) / 2 and x[O] = b (P - Q) / 2. The map phi satisfies
phi^T phi = 2 I, so all three sums are phi^-1(sum_Cl(6,0)(phi(x), phi(y))).
"""
import numpy as np

from oracle import ga_oracle as O

M61, M60 = (1,) * 6 + (-1,), (1,) * 6


def bsign(p, q, metric):
    """sign of e_p e_q (the oracle's rule: reorder parity and the metric)."""
    s = 0
    for a in range(7):
        if (p >> a) & 1:
            s += bin(q & ((1 << a) - 1)).count("1")
    m = 1
    for a in range(7):
        if (p >> a) & 1 and (q >> a) & 1:
            m *= metric[a]
    return (-1) ** s * m


def tables():
    E, A, B = [], [], []
    for k in range(64):
        blade, sign = 0, 1
        for i in range(6):
            if (k >> i) & 1:
                for g in (1 << i, 1 << 6):
                    sign *= bsign(blade, g, M61)
                    blade ^= g
        o = blade ^ 127
        E.append(blade)
        A.append(sign)
        B.append(sign * bsign(o, 127, M61))
    return np.array(E), np.array(A, float), np.array(B, float)


def phi(x):
    E, A, B = tables()
    xe, xo = x[:, E], x[:, E ^ 127]
    return A * xe + B * xo, A * xe - B * xo


def phi_inv(P, Q):
    E, A, B = tables()
    x = np.zeros((P.shape[0], 128))
    x[:, E] = A * (P + Q) / 2
    x[:, E ^ 127] = B * (P - Q) / 2
    return x


def test_tables_are_a_bijection():
    E, _, _ = tables()
    assert sorted(list(E) + list(E ^ 127)) == list(range(128))
    assert all(bin(e).count("1") % 2 == 0 for e in E)


def test_cl61_sums_through_two_cl60_sums():
    rng = np.random.default_rng(1)
    a, b, g = (rng.standard_normal((5, 128)) for _ in range(3))
    ref = O.forward_backward("gp", 7, M61, a, b, g)
    for mode, x, y, r in (("fwd", a, b, ref[0]), ("grad_a", b, g, ref[1]), ("grad_b", a, g, ref[2])):
        (px, qx), (py, qy) = phi(x), phi(y)
        out = phi_inv(O.product("gp", mode, 6, M60, px, py), O.product("gp", mode, 6, M60, qx, qy))
        assert np.abs(out - r).max() <= 1e-12 * np.abs(r).max(), mode
