"""``CliffordAlgebra``: the reference's public class
(``src/cliffordcuda/algebra.py:88-385``) on the B200 kernels.

Bound at construction: ``metric`` (length-n iterable of {-1, 0, +1}), ``n``,
``dim = 2**n``, ``device`` and ``dtype`` (always float32). Product methods take
two ``(batch, dim)`` multivectors and return one; the rotor methods take a
bivector ``(1, C(n, 2))`` in lex-pair order.
"""
from __future__ import annotations

import torch

from . import _validate
from . import products as _p


class CliffordAlgebra:
    def __init__(self, metric, device="cuda"):
        metric = _validate._check_metric(metric)
        self.metric = metric
        self.n = len(metric)
        self.dim = 1 << self.n
        self.device = _validate._check_device(device)
        # fp32 only, as in the reference (algebra.py:98).
        self.dtype = torch.float32
        self._num_basis_biv = self.n * (self.n - 1) // 2
        # the reference's rotor range, n >= 7 (algebra.py:106-113).
        self._rotor_supported = self.n >= 7
        self._rotor = None

    # ── products (algebra.py:143-171) ────────────────────────────────
    def _check2(self, a, b):
        _validate._check_mv(a, "a", self.dim, self.device, self.dtype)
        _validate._check_mv(b, "b", self.dim, self.device, self.dtype)

    def geom_prod(self, a, b):
        self._check2(a, b)
        return _p.geom_prod(a, b, metric=self.metric)

    def wedge_prod(self, a, b):
        self._check2(a, b)
        return _p.wedge_prod(a, b, metric=self.metric)

    def inner_prod(self, a, b):
        self._check2(a, b)
        return _p.inner_prod(a, b, metric=self.metric)

    def left_contraction(self, a, b):
        self._check2(a, b)
        return _p.left_contract(a, b, metric=self.metric)

    def right_contraction(self, a, b):
        self._check2(a, b)
        return _p.right_contract(a, b, metric=self.metric)

    def regressive_prod(self, a, b):
        if 0 in self.metric:
            raise ValueError(
                "regressive_prod is undefined for degenerate metrics "
                "(any 0 in the metric makes the pseudoscalar non-invertible).")
        self._check2(a, b)
        return _p.regressive_prod(a, b, metric=self.metric)

    # ── sign-vector elementwise ops (algebra.py:195-336) ─────────────
    # One-pass multiplies by a per-blade sign or weight vector; they run as
    # torch elementwise ops on the device (not part of the kernel library).
    def _grades(self):
        if not hasattr(self, "_grade_vec"):
            idx = torch.arange(self.dim, device=self.device)
            k = torch.zeros(self.dim, device=self.device, dtype=torch.long)
            for t in range(self.n):
                k += (idx >> t) & 1
            self._grade_vec = k
        return self._grade_vec

    def reverse(self, x):
        """Reversion: grade k -> (-1)^(k(k-1)/2)."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        k = self._grades()
        return x * torch.where(((k * (k - 1) // 2) % 2) == 1, -1.0, 1.0).to(self.dtype)

    def grade_involution(self, x):
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        k = self._grades()
        return x * torch.where((k % 2) == 1, -1.0, 1.0).to(self.dtype)

    def clifford_conjugation(self, x):
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        k = self._grades()
        return x * torch.where(((k * (k + 1) // 2) % 2) == 1, -1.0, 1.0).to(self.dtype)

    def grade_projection(self, x, grade):
        if not 0 <= grade <= self.n:
            raise ValueError(f"grade must be in [0, {self.n}] for n={self.n}; got {grade}")
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return x * (self._grades() == grade).to(self.dtype)

    def _metric_weights(self):
        idx = torch.arange(self.dim, device=self.device)
        w = torch.ones(self.dim, device=self.device)
        for t in range(self.n):
            w = w * torch.where(((idx >> t) & 1).bool(), float(self.metric[t]), 1.0)
        return w.to(self.dtype)

    def norm_sq(self, x, compile=False):
        """<x x~>_0 = sum_b x_b^2 prod_{i in b} metric[i]; shape (batch,)."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return (x * x * self._metric_weights()).sum(-1)

    def dual(self, x, compile=False):
        """x I^-1: a signed reversal of the coefficients (non-degenerate only)."""
        if 0 in self.metric:
            raise ValueError(
                "dual is undefined for degenerate metrics (any 0 in the "
                "metric makes the pseudoscalar I non-invertible).")
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        n, full = self.n, self.dim - 1
        i_sq = (-1) ** (n * (n - 1) // 2)
        for m in self.metric:
            i_sq *= m
        idx = torch.arange(self.dim, device=self.device)
        a = full ^ idx
        swaps = torch.zeros(self.dim, device=self.device, dtype=torch.long)
        for t in range(n):
            swaps += t * ((a >> t) & 1)
        signs = float(i_sq) * torch.where((swaps % 2) == 1, -1.0, 1.0) * \
            self._metric_weights().index_select(0, a)
        return x.flip(-1) * signs.to(self.dtype)

    # ── rotors (algebra.py:337-373) ──────────────────────────────────
    def _check_rotor_supported(self):
        if not self._rotor_supported:
            raise ValueError(
                f"rotor application requires n >= 7 (ppr = 2^(n-2) must be "
                f"at least 32 = warp size); got n={self.n}")

    def _rotor_engine(self):
        if self._rotor is None:
            from .rotor import RotorEngine
            self._rotor = RotorEngine(self.n, self.device)
        return self._rotor

    def compile_bivector(self, bivector):
        """Compile a bivector into the rotor handle that ``apply_rotor``
        consumes (opaque; here the blade-minor matrices of
        Rm = expm(2 (M - M^T)))."""
        self._check_rotor_supported()
        _validate._check_bivector(bivector, self.n, self._num_basis_biv, self.device, self.dtype)
        return self._rotor_engine().compile(bivector)

    def apply_rotor(self, cs, x):
        """y = R~ x R for a compiled rotor (Euclidean sandwich; the metric is
        not used on the rotor path, as in the reference)."""
        self._check_rotor_supported()
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return self._rotor_engine().apply(cs, x)

    def apply_bivector(self, bivector, x):
        """``apply_rotor(compile_bivector(bivector), x)``."""
        return self.apply_rotor(self.compile_bivector(bivector), x)

    def to(self, device):
        return CliffordAlgebra(self.metric, device=device)

    def __repr__(self):
        p = sum(1 for m in self.metric if m == 1)
        q = sum(1 for m in self.metric if m == -1)
        r = sum(1 for m in self.metric if m == 0)
        return (f"CliffordAlgebra(metric={list(self.metric)}, Cl({p}, {q}, {r}), "
                f"n={self.n}, dim={self.dim}, device={self.device})")
