"""Failure detection on the GPU without a fault: a kernel's bounded wait on a
barrier that nothing completes gives up, the failure is reported as a status
by cb_device_status, and the context keeps working afterwards."""
import ctypes

import pytest
import torch

import cliffordcuda_b200 as cc
from cliffordcuda_b200 import _lib

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_status_and_context_survives():
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.cb_device_status(stream) == 0
    assert lib.cb_selftest_bounded_wait(2000, stream) == 0
    assert lib.cb_device_status(stream) == 4          # CB_ERR_DEVICE
    assert b"bounded wait" in lib.cb_last_error()
    assert lib.cb_device_status(stream) == 0          # the flag was cleared
    a = torch.randn(8, 256, device="cuda")
    c = cc.geom_prod(a, a)                            # the context still works
    assert torch.isfinite(c).all()
    with pytest.raises(_lib.CliffordNativeError):
        lib.cb_selftest_bounded_wait(10, stream)
        _lib.device_status()
