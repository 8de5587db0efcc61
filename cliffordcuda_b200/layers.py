"""``nn.Module`` layers (reference ``src/cliffordcuda/layers.py:30-108``).

Product layers hold a learnable ``weight`` of shape ``(1, 2^n)`` and compute
``product(x, weight)`` (input on the left, weight on the right). The weight
is shared across the batch, so the product is a dense contraction
``y = x M(w)`` with ``M(w)[i, k] = s(i, i^k) w[i^k]``; see ``layer_ops``.
``RotorLayer`` holds ``bivector`` ``(1, C(n, 2))`` and computes R~ x R.
Parameter names match the reference so its ``state_dict`` files load.
"""
import torch
import torch.nn as nn

from . import _validate, layer_ops


class _ProductLayer(nn.Module):
    _op: str = None
    _method: str = None

    def __init__(self, cl):
        super().__init__()
        self.cl = cl
        self.weight = nn.Parameter(torch.randn(1, cl.dim, device=cl.device, dtype=cl.dtype))

    def forward(self, x):
        _validate._check_mv(x, "x", self.cl.dim, self.cl.device, self.cl.dtype)
        if self._op == "reg" and 0 in self.cl.metric:
            raise ValueError(
                "regressive_prod is undefined for degenerate metrics "
                "(any 0 in the metric makes the pseudoscalar non-invertible).")
        return layer_ops.layer_product(self._op, x, self.weight, self.cl.n, self.cl.metric)

    def extra_repr(self):
        return f"n={self.cl.n}, dim={self.cl.dim}, op={self._method}"


class GeometricProductLayer(_ProductLayer):
    _op, _method = "gp", "geom_prod"


class WedgeProductLayer(_ProductLayer):
    _op, _method = "wedge", "wedge_prod"


class InnerProductLayer(_ProductLayer):
    _op, _method = "inner", "inner_prod"


class LeftContractionLayer(_ProductLayer):
    _op, _method = "lc", "left_contraction"


class RightContractionLayer(_ProductLayer):
    _op, _method = "rc", "right_contraction"


class RegressiveProductLayer(_ProductLayer):
    _op, _method = "reg", "regressive_prod"


class RotorLayer(nn.Module):
    """Learnable rotor (reference layers.py:79-108): recompiled every forward
    in train(), compiled once and cached in eval(). Requires n >= 7."""

    def __init__(self, cl):
        super().__init__()
        if cl.n < 7:
            raise ValueError(f"RotorLayer requires n>=7 (rotor support); got n={cl.n}")
        self.cl = cl
        nb = cl.n * (cl.n - 1) // 2
        self.bivector = nn.Parameter(torch.randn(1, nb, device=cl.device, dtype=cl.dtype))
        self._cs = None

    def train(self, mode=True):
        self._cs = None
        return super().train(mode)

    def forward(self, x):
        if self.training:
            return self.cl.apply_bivector(self.bivector, x)
        if self._cs is None:
            with torch.no_grad():
                self._cs = self.cl.compile_bivector(self.bivector)
        return self.cl.apply_rotor(self._cs, x)

    def extra_repr(self):
        return f"n={self.cl.n}, dim={self.cl.dim}, num_basis_biv={self.bivector.shape[-1]}"
