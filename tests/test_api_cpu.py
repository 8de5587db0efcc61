"""Host-side API behaviour without a GPU: validation errors match the
reference's (ValueError at the boundary) and nothing falls back to the CPU."""
import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _validate
from cliffordcuda_b200.products import _normalize_metric, metric_masks


def test_metric_validation():
    with pytest.raises(ValueError):
        _validate._check_metric([1, 2])
    with pytest.raises(ValueError):
        _validate._check_metric([])
    with pytest.raises(ValueError):
        _validate._check_metric(5)
    assert _validate._check_metric([1, -1, 0]) == (1, -1, 0)


def test_cpu_device_rejected():
    with pytest.raises(ValueError):
        cc.CliffordAlgebra([1] * 5, device="cpu")


def test_free_functions_reject_cpu_tensors():
    a = torch.randn(2, 32)
    for f in (cc.geom_prod, cc.wedge_prod, cc.inner_prod, cc.left_contract,
              cc.right_contract, cc.regressive_prod):
        with pytest.raises(ValueError):
            f(a, a)


def test_free_function_shape_checks():
    with pytest.raises(ValueError):
        cc.geom_prod(torch.randn(2, 16), torch.randn(2, 16))      # n < 5
    with pytest.raises(ValueError):
        cc.geom_prod(torch.randn(2, 48), torch.randn(2, 48))      # not a power of two
    with pytest.raises(ValueError):
        cc.geom_prod(torch.randn(2, 32), torch.randn(3, 32))      # shape mismatch


def test_metric_masks():
    assert metric_masks((1, -1, 0, -1)) == (0b1010, 0b0100)
    assert _normalize_metric(3, None) == (1, 1, 1)
    with pytest.raises(ValueError):
        _normalize_metric(3, (1, 1))


def test_check_mv_messages():
    dev = torch.device("cuda", 0)
    with pytest.raises(ValueError, match="2D"):
        _validate._check_mv(torch.zeros(3), "x", 32, dev, torch.float32)
    with pytest.raises(ValueError, match="last dim"):
        _validate._check_mv(torch.zeros(2, 16), "x", 32, dev, torch.float32)
    with pytest.raises(ValueError, match="device"):
        _validate._check_mv(torch.zeros(2, 32), "x", 32, dev, torch.float32)
