"""cb_rotor_apply_bwd_noalloc: the rotor backward for callers that cannot
allocate device memory (it keeps its per-CTA partial sums in a fixed array
inside the library instead of a caller workspace). Checked through the C ABI
against cb_rotor_apply_bwd on two calls in a row, so stale contents of the
shared array from the first call would show up in the second. This file is
named to be collected last."""
import ctypes

import numpy as np
import pytest
import torch

from cliffordcuda_b200 import _lib
from tests.helpers import REL_L2_TOL, rel_l2

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _compiled(n, seed):
    lib = _lib.load()
    cs_n, st_n = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(lib.cb_rotor_sizes(n, ctypes.byref(cs_n), ctypes.byref(st_n)), "sizes")
    gen = torch.Generator(device=DEV).manual_seed(seed)
    beta = 0.2 * torch.randn(n * (n - 1) // 2, device=DEV, generator=gen)
    cs = torch.empty(cs_n.value, device=DEV)
    state = torch.empty(st_n.value, device=DEV, dtype=torch.float64)
    stream = _lib.stream_of(cs)
    _lib.check(lib.cb_rotor_compile(_lib.ptr(beta), n, _lib.ptr(cs), _lib.ptr(state), stream),
               "compile")
    return cs


def _both(n, batch, seed):
    lib = _lib.load()
    cs = _compiled(n, seed)
    gen = torch.Generator(device=DEV).manual_seed(seed + 1)
    x = torch.randn(batch, 1 << n, device=DEV, generator=gen)
    g = torch.randn(batch, 1 << n, device=DEV, generator=gen)
    stream = _lib.stream_of(x)
    dx_ref, dcs_ref = torch.empty_like(x), torch.empty_like(cs)
    wb = ctypes.c_int64()
    _lib.check(lib.cb_rotor_workspace_bytes(n, batch, ctypes.byref(wb)), "workspace")
    ws = torch.empty(wb.value, device=DEV, dtype=torch.uint8)
    _lib.check(lib.cb_rotor_apply_bwd(_lib.ptr(cs), _lib.ptr(x), _lib.ptr(g), _lib.ptr(dx_ref),
                                      _lib.ptr(dcs_ref), batch, n, _lib.ptr(ws), wb.value,
                                      stream), "apply_bwd")
    dx, dcs = torch.full_like(x, float("nan")), torch.full_like(cs, float("nan"))
    _lib.check(lib.cb_rotor_apply_bwd_noalloc(_lib.ptr(cs), _lib.ptr(x), _lib.ptr(g),
                                              _lib.ptr(dx), _lib.ptr(dcs), batch, n, stream),
               "apply_bwd_noalloc")
    torch.cuda.synchronize()
    return (dx.cpu().numpy(), dcs.cpu().numpy()), (dx_ref.cpu().numpy(), dcs_ref.cpu().numpy())


@pytest.mark.parametrize("n,batches", [(8, (300_000, 1_000)), (7, (5_000, 200_000)),
                                       (8, (2_097_152, 3))])
def test_noalloc_matches_workspace_entry_point_twice(n, batches):
    for call, batch in enumerate(batches):
        (dx, dcs), (dx_ref, dcs_ref) = _both(n, batch, seed=10 * n + call)
        assert np.isfinite(dx).all() and np.isfinite(dcs).all()
        assert rel_l2(dx, dx_ref) <= REL_L2_TOL, f"call {call}: dx"
        assert rel_l2(dcs, dcs_ref) <= REL_L2_TOL, f"call {call}: dcs"
    _lib.device_status(DEV)


def test_noalloc_rejects_unsupported_n():
    lib = _lib.load()
    null = ctypes.c_void_p(0)
    assert lib.cb_rotor_apply_bwd_noalloc(null, null, null, null, null, 1, 9, null) == 3
    assert b"n = 7 and 8" in lib.cb_last_error()
