"""CPU oracle for the multivector-product hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of bench.py
import this module, and only as the checker or as the timed CPU reference.
The shipped library (cliffordcuda_b200/) never imports it.

Three restatements of the reference live here:

* ``ga_oracle.c`` (wrapped below via ctypes): double-precision products,
  regressive product and rotor outermorphism. See that file's header for the
  reference file:line of each function.
* ``EinsumProduct``: a torch port of the reference's CPU path
  ``_shared/_einsum_refs.py:26-124`` (outer product x signed mask, then a
  scatter-add to k = i ^ j). It is what ``bench.py --impl reference`` times on
  the host cores, because the reference's own copy of that code cannot travel
  to the GPU box.
* ``givens_chain_apply``: the reference's rotor arithmetic step by step --
  the Givens factorisation of ``givens_factor.cu:7-59`` and the rotation
  sweep of ``givens_apply_mb_perm_packed.cu:33-66`` with the pair tables of
  ``_utils/core.py:5-50``. It pins that the blade-minor form used by the C
  oracle (and by the CUDA path) equals the reference's chain.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libga_oracle.so")

OPS = {"gp": 0, "wedge": 1, "inner": 2, "lc": 3, "rc": 4}
MODES = {"fwd": 0, "grad_a": 1, "grad_b": 2}

_lib = None


def build():
    """Compile ga_oracle.c into oracle/_build/ (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        dp = ctypes.POINTER(ctypes.c_double)
        ip = ctypes.POINTER(ctypes.c_int)
        L.orc_sign.restype = ctypes.c_int
        L.orc_sign.argtypes = [ctypes.c_int, ip, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_sign_table.argtypes = [ctypes.c_int, ctypes.c_int, ip,
                                     ctypes.POINTER(ctypes.c_int8)]
        L.orc_product.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ip,
                                  ctypes.c_int64, dp, dp, dp]
        L.orc_product_range.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ip,
                                        ctypes.c_int64, dp, dp, dp, ctypes.c_uint32,
                                        ctypes.c_uint32]
        L.orc_regressive_fwd.argtypes = [ctypes.c_int, ip, ctypes.c_int64, dp, dp, dp]
        L.orc_regressive_bwd.argtypes = [ctypes.c_int, ip, ctypes.c_int64,
                                         dp, dp, dp, dp, dp]
        L.orc_rotor_matrix.argtypes = [ctypes.c_int, dp, dp]
        L.orc_rotor_blade_matrix.argtypes = [ctypes.c_int, dp, dp]
        L.orc_rotor_apply_matrix.argtypes = [ctypes.c_int, dp, ctypes.c_int64, dp, dp]
        _lib = L
    return _lib


def _dptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _metric_arr(metric):
    return (ctypes.c_int * len(metric))(*[int(m) for m in metric])


def _rows(x, D):
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float64))
    return x.reshape(-1, D)


def _split(batch, threads):
    threads = max(1, min(threads, batch))
    step = (batch + threads - 1) // threads
    return [(s, min(batch, s + step)) for s in range(0, batch, step)]


def _threaded(batch, threads, fn):
    threads = threads or os.cpu_count() or 1
    if batch == 0:
        return
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(fn, _split(batch, threads)))


def sign_table(n, metric, op="gp"):
    """(D, D) int8 signed-mask table of `op` (geom_prod.py:44-74 x mask)."""
    D = 1 << n
    out = np.empty((D, D), dtype=np.int8)
    lib().orc_sign_table(OPS[op], n, _metric_arr(metric),
                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)))
    return out


def product(op, mode, n, metric, x, y, threads=None):
    """Double-precision bilinear sum of the reference (see ga_oracle.c).

    op in gp|wedge|inner|lc|rc; mode in fwd|grad_a|grad_b with
    fwd: (x, y) = (a, b);  grad_a: (x, y) = (b, g);  grad_b: (x, y) = (a, g).
    For the regressive product use `regressive_fwd` / `regressive_bwd`.
    """
    D = 1 << n
    x = _rows(x, D)
    y = _rows(y, D)
    out = np.empty_like(x)
    m = _metric_arr(metric)
    L = lib()

    if n >= 11:
        # no (D, D) table; the output blades are split over the threads
        nt = threads or os.cpu_count() or 1
        step = (D + nt - 1) // nt

        def run_k(k0):
            L.orc_product_range(OPS[op], MODES[mode], n, m, x.shape[0], _dptr(x), _dptr(y),
                                _dptr(out), k0, min(D, k0 + step))

        if x.shape[0]:
            with ThreadPoolExecutor(nt) as ex:
                list(ex.map(run_k, range(0, D, step)))
        return out

    def run(rng):
        s, e = rng
        L.orc_product(OPS[op], MODES[mode], n, m, e - s,
                      _dptr(x[s:e]), _dptr(y[s:e]), _dptr(out[s:e]))

    _threaded(x.shape[0], threads, run)
    return out


def forward_backward(op, n, metric, a, b, g, threads=None):
    """(c, grad_a, grad_b) of op(a, b) for upstream gradient g, in double."""
    if op == "reg":
        return (regressive_fwd(n, metric, a, b),) + tuple(regressive_bwd(n, metric, a, b, g))
    c = product(op, "fwd", n, metric, a, b, threads)
    ga = product(op, "grad_a", n, metric, b, g, threads)
    gb = product(op, "grad_b", n, metric, a, g, threads)
    return c, ga, gb


def regressive_fwd(n, metric, a, b):
    D = 1 << n
    a, b = _rows(a, D), _rows(b, D)
    out = np.empty_like(a)
    lib().orc_regressive_fwd(n, _metric_arr(metric), a.shape[0], _dptr(a),
                             _dptr(b), _dptr(out))
    return out


def regressive_bwd(n, metric, a, b, g):
    D = 1 << n
    a, b, g = _rows(a, D), _rows(b, D), _rows(g, D)
    ga, gb = np.empty_like(a), np.empty_like(a)
    lib().orc_regressive_bwd(n, _metric_arr(metric), a.shape[0], _dptr(a),
                             _dptr(b), _dptr(g), _dptr(ga), _dptr(gb))
    return ga, gb


# ------------------------------------------------------------------ rotor --

def rotor_matrix(n, beta):
    """Rm = expm(2 (M - M^T)) in double (eigh_exp.cu:270-322 restated)."""
    beta = np.ascontiguousarray(np.asarray(beta, dtype=np.float64).reshape(-1))
    Rm = np.empty((n, n), dtype=np.float64)
    lib().orc_rotor_matrix(n, _dptr(beta), _dptr(Rm))
    return Rm


def rotor_blade_matrix(n, Rm):
    """C[I, J] = det(Rm[I, J]) on equal-grade blade pairs; y = x @ C."""
    D = 1 << n
    Rm = np.ascontiguousarray(Rm, dtype=np.float64)
    C = np.empty((D, D), dtype=np.float64)
    lib().orc_rotor_blade_matrix(n, _dptr(Rm), _dptr(C))
    return C


def rotor_apply(n, beta, x, threads=None):
    """y = R~ x R (Euclidean outermorphism of Rm^T), double precision."""
    D = 1 << n
    C = rotor_blade_matrix(n, rotor_matrix(n, beta))
    x = _rows(x, D)
    y = np.empty_like(x)
    L = lib()

    def run(rng):
        s, e = rng
        L.orc_rotor_apply_matrix(n, _dptr(C), e - s, _dptr(x[s:e]), _dptr(y[s:e]))

    _threaded(x.shape[0], threads, run)
    return y


def givens_chain_apply(n, Rm, x):
    """The reference's rotor arithmetic, step by step, in double.

    Factorisation (givens_factor.cu:7-59): sweep planes (p, q) in lex order,
    c = A[p,p]/r, s_raw = -A[q,p]/r, rotate rows p and q of A; record
    (c, -s_raw) at slot n_rot-1-count. Apply (givens_apply_mb_perm_packed.cu:
    33-66): for rot = n_rot-1 .. 0 take plane (p, q) = reversed-lex[rot]
    (_utils/core.py:5-50) and for every blade i with bit p set and bit q clear,
    j = i ^ (1<<p | 1<<q): x_i' = c x_i + s sig x_j, x_j' = -s sig x_i + c x_j.
    """
    A = np.array(Rm, dtype=np.float64)
    n_rot = n * (n - 1) // 2
    cs = np.zeros((n_rot, 2))
    count = 0
    for p in range(n - 1):
        for q in range(p + 1, n):
            a, bv = A[p, p], A[q, p]
            r = math.sqrt(a * a + bv * bv)
            inv_r = 1.0 / max(r, 1e-300)
            c, s_raw = a * inv_r, -bv * inv_r
            cs[n_rot - 1 - count] = (c, -s_raw)
            Ap, Aq = A[p].copy(), A[q].copy()
            A[p] = c * Ap - s_raw * Aq
            A[q] = s_raw * Ap + c * Aq
            count += 1
    pq_rev = list(reversed([(p, q) for p in range(n - 1) for q in range(p + 1, n)]))
    D = 1 << n
    y = np.array(x, dtype=np.float64).reshape(-1, D).copy()
    for rot in range(n_rot - 1, -1, -1):
        p, q = pq_rev[rot]
        c, s = cs[rot]
        mask = (1 << p) | (1 << q)
        for i in range(D):
            if ((i >> p) & 1) and not ((i >> q) & 1):
                j = i ^ mask
                removal = bin(i).count("1") - 1 - bin(i & ((1 << p) - 1)).count("1")
                insert = bin(i >> (q + 1)).count("1")
                sig = -1.0 if ((removal + insert) & 1) else 1.0
                xi, xj = y[:, i].copy(), y[:, j].copy()
                y[:, i] = c * xi + s * sig * xj
                y[:, j] = -s * sig * xi + c * xj
    return y


def _rotor_C_torch(n, beta_t):
    """C(beta) in torch fp64, differentiable: C[I, J] = det Rm[I, J] on
    equal-grade blade pairs, Rm = matrix_exp(2 (M - M^T)), M[p, q] = beta_pq
    for p < q in lex-pair order (reference algebra.py:127, eigh_exp.cu:270-322)."""
    import torch
    D = 1 << n
    iu = torch.triu_indices(n, n, offset=1)
    M = torch.zeros(n, n, dtype=torch.float64).index_put((iu[0], iu[1]), beta_t)
    Rm = torch.linalg.matrix_exp(2.0 * (M - M.T))
    cols = []
    for J in range(D):
        col = []
        for I in range(D):
            if bin(I).count("1") != bin(J).count("1"):
                col.append(torch.zeros((), dtype=torch.float64))
            elif I == 0:
                col.append(torch.ones((), dtype=torch.float64))
            else:
                ri = [t for t in range(n) if (I >> t) & 1]
                ci = [t for t in range(n) if (J >> t) & 1]
                col.append(torch.linalg.det(Rm[ri][:, ci]))
        cols.append(torch.stack(col))
    return torch.stack(cols, dim=1)  # C[I, J]


def rotor_grads_torch(n, beta, x, g):
    """fp64 autograd truth for the rotor: (y, dL/dx, dL/dbeta) with
    L = <g, y>, y = x C(Rm), Rm = torch.linalg.matrix_exp(2 (M - M^T))."""
    import torch
    D = 1 << n
    beta_t = torch.tensor(np.asarray(beta, dtype=np.float64).reshape(-1), requires_grad=True)
    x_t = torch.tensor(np.asarray(x, dtype=np.float64).reshape(-1, D), requires_grad=True)
    C = _rotor_C_torch(n, beta_t)
    y = x_t @ C
    g_t = torch.tensor(np.asarray(g, dtype=np.float64).reshape(-1, D))
    (y * g_t).sum().backward()
    return y.detach().numpy(), x_t.grad.numpy(), beta_t.grad.numpy()


def rotor_dbeta_from_G(n, beta, G):
    """dL/dbeta for L = <g, x C(beta)> summed over a batch, given only
    G = sum over rows of x^T g (D x D, fp64): L = sum_IJ C[I, J] G[I, J], so
    the batch enters through G alone and large batches cost one GEMM."""
    import torch
    beta_t = torch.tensor(np.asarray(beta, dtype=np.float64).reshape(-1), requires_grad=True)
    C = _rotor_C_torch(n, beta_t)
    (C * torch.as_tensor(np.asarray(G, dtype=np.float64))).sum().backward()
    return beta_t.grad.numpy()


def layer_dw_from_G(op, n, metric, G):
    """Weight gradient of a product layer y = op(x, w) summed over the batch,
    from G = sum over rows of x^T dy (D x D, fp64): the reference's
    expand_as formulation (layers.py:43-47) sums grad_b(x, dy) over rows, and
    grad_b[k] = sum_i s(i, k) x[i] dy[i ^ k], so dw[k] = sum_i s(i, k) G[i, i ^ k].
    Products gp, wedge, inner, lc, rc (not the regressive one)."""
    D = 1 << n
    S = sign_table(n, metric, op).astype(np.float64)   # S[P, Q] with (P, Q) = (i, k)
    i = np.arange(D).reshape(-1, 1)
    k = np.arange(D).reshape(1, -1)
    G = np.asarray(G, dtype=np.float64)
    return (S * G[i, i ^ k]).sum(axis=0)


# ---------------------------------------------------- torch einsum port --

class EinsumProduct:
    """Torch restatement of the reference CPU path (_einsum_refs.py:26-124):
    outer(A, B) * signs, scatter-added to k = i ^ j. Backward by autograd."""

    def __init__(self, op, n, metric, dtype=None):
        import torch
        self.torch = torch
        dtype = dtype or torch.float32
        self.op, self.n, self.D = op, n, 1 << n
        D = self.D
        i = torch.arange(D)
        self.indices = (i.view(-1, 1) ^ i.view(1, -1)).reshape(-1)
        base = "wedge" if op == "reg" else op
        self.signs = torch.from_numpy(sign_table(n, metric, base).astype(np.float32)).to(dtype)
        if op == "reg":
            full = D - 1
            sig = sign_table(n, metric, "gp")
            isq = float(sig[full, full])
            self.comp = i ^ full
            self.ds = torch.from_numpy(
                (sig[(i ^ full).numpy(), full] / isq).astype(np.float32)).to(dtype)

    def _wedge_like(self, A, B):
        torch = self.torch
        outer = torch.einsum("...i,...j->...ij", A, B) * self.signs
        flat = outer.reshape(*outer.shape[:-2], -1)
        idx = self.indices.expand_as(flat)
        out = torch.zeros(*flat.shape[:-1], self.D, dtype=A.dtype)
        return out.scatter_add(-1, idx, flat)

    def __call__(self, A, B):
        if self.op == "reg":
            d = lambda x: x.index_select(-1, self.comp) * self.ds
            return d(self._wedge_like(d(A), d(B)))
        return self._wedge_like(A, B)


# ------------------------------------------------------------ blade maps --

def _grades(n):
    return np.array([bin(i).count("1") for i in range(1 << n)])


def blade_map(kind, n, metric, x, grade=None):
    """Per-blade maps of CliffordAlgebra in float64 (reference
    src/cliffordcuda/algebra.py): reverse (:195-206, (-1)^(k(k-1)/2)),
    involute (:278-286, (-1)^k), conjugate (:288-296, (-1)^(k(k+1)/2)),
    grade (:298-307, keep grade `grade`), dual (:208-266: out[m] = s(a) x[a],
    a = ~m, s(a) = (1/I^2) (-1)^(sum of a's generator positions) prod_{t in a}
    metric[t]) and dual_t, the dual's transpose (out[m] = s(m) x[~m])."""
    D = 1 << n
    x = np.asarray(x, dtype=np.float64).reshape(-1, D)
    k = _grades(n)
    if kind == "reverse":
        return x * np.where((k * (k - 1) // 2) % 2 == 1, -1.0, 1.0)
    if kind == "involute":
        return x * np.where(k % 2 == 1, -1.0, 1.0)
    if kind == "conjugate":
        return x * np.where((k * (k + 1) // 2) % 2 == 1, -1.0, 1.0)
    if kind == "grade":
        return x * (k == grade)
    if kind in ("dual", "dual_t"):
        if 0 in metric:
            raise ValueError("dual needs a non-degenerate metric")
        i_sq = (-1) ** (n * (n - 1) // 2) * int(np.prod(metric))
        idx = np.arange(D)
        a = (D - 1) ^ idx if kind == "dual" else idx
        pos = np.zeros(D, dtype=np.int64)
        mprod = np.ones(D)
        for t in range(n):
            bit = (a >> t) & 1
            pos += t * bit
            mprod *= np.where(bit == 1, float(metric[t]), 1.0)
        s = i_sq * np.where(pos % 2 == 1, -1.0, 1.0) * mprod
        return x[:, (D - 1) ^ idx] * s
    raise ValueError(kind)


def norm_sq(n, metric, x):
    """sum_b x_b^2 prod_{t in b} metric[t], float64 (algebra.py:309-336)."""
    D = 1 << n
    x = np.asarray(x, dtype=np.float64).reshape(-1, D)
    w = np.ones(D)
    idx = np.arange(D)
    for t in range(n):
        w *= np.where((idx >> t) & 1 == 1, float(metric[t]), 1.0)
    return (x * x * w).sum(-1)
