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
from . import blade_maps as _maps
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

    # ── per-blade maps and the norm (algebra.py:195-336) ─────────────
    # One pass each on the native kernels (cb_blade_map, cb_norm_sq), with
    # autograd; `compile` is accepted for API compatibility and has no effect
    # (the kernel already makes a single memory pass).
    def reverse(self, x):
        """Reversion: grade k -> (-1)^(k(k-1)/2)."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.blade_map("reverse", x, self.metric)

    def grade_involution(self, x):
        """Grade involution: grade k -> (-1)^k."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.blade_map("involute", x, self.metric)

    def clifford_conjugation(self, x):
        """Clifford conjugation: grade k -> (-1)^(k(k+1)/2)."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.blade_map("conjugate", x, self.metric)

    def grade_projection(self, x, grade):
        """Keep the grade-`grade` coefficients, zero the others (same shape)."""
        if not 0 <= grade <= self.n:
            raise ValueError(f"grade must be in [0, {self.n}] for n={self.n}; got {grade}")
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.blade_map("grade", x, self.metric, grade)

    def norm_sq(self, x, compile=False):
        """<x x~>_0 = sum_b x_b^2 prod_{i in b} metric[i]; shape (batch,)."""
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.norm_sq(x, self.metric)

    def dual(self, x, compile=False):
        """x I^-1: a signed reversal of the coefficients (non-degenerate only)."""
        if 0 in self.metric:
            raise ValueError(
                "dual is undefined for degenerate metrics (any 0 in the "
                "metric makes the pseudoscalar I non-invertible).")
        _validate._check_mv(x, "x", self.dim, self.device, self.dtype)
        return _maps.blade_map("dual", x, self.metric)

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
