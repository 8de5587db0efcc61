"""Shared-weight product layers: y = op(x, w) with one weight row for the
whole batch (reference layers.py:43-47, which materialised
``w.expand_as(x)`` and ran the batch-by-batch kernel)."""
from __future__ import annotations

from . import products as _p


def layer_product(op, x, weight, n, metric):
    w = weight.expand_as(x).contiguous()
    return _p._product(op, x, w, metric)
