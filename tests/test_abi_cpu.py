"""The C-ABI library loads, exports every symbol include/*.h declares, and
rejects bad arguments before touching a device. No GPU needed."""
import ctypes
import glob
import os
import re

import pytest

from cliffordcuda_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NULL = ctypes.c_void_p(0)


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        for m in re.finditer(r"CB_API\s+[\w\s\*]+?\b(cb_\w+)\s*\(", open(h).read()):
            syms.add(m.group(1))
    return syms


def test_header_declares_entry_points():
    assert {"cb_bilinear", "cb_bilinear_bwd", "cb_last_error", "cb_version"} <= declared_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_version():
    assert _lib.load().cb_version() >= 100


@pytest.mark.parametrize("args,code", [
    ((9, 0, 8, 1), 1),        # op out of range
    ((0, 7, 8, 1), 1),        # mode out of range
    ((0, 0, 17, 1), 3),       # n too large
    ((0, 0, 0, 1), 3),        # n too small
    ((0, 0, 8, -1), 1),       # negative batch
    ((0, 0, 8, 4), 1),        # null pointers
])
def test_bad_arguments_rejected(args, code):
    op, mode, n, batch = args
    lib = _lib.load()
    assert lib.cb_bilinear(op, mode, NULL, NULL, NULL, batch, n, 0, 0, NULL) == code
    assert lib.cb_last_error()


def test_bad_metric_masks_rejected():
    lib = _lib.load()
    assert lib.cb_bilinear(0, 0, NULL, NULL, NULL, 1, 5, 1 << 6, 0, NULL) == 1   # bit past n
    assert lib.cb_bilinear(0, 0, NULL, NULL, NULL, 1, 5, 1, 1, NULL) == 1        # both masks
    assert lib.cb_bilinear(5, 0, NULL, NULL, NULL, 1, 5, 0, 2, NULL) == 1        # reg, degenerate
    assert b"degenerate" in lib.cb_last_error()


def test_aliasing_rejected():
    lib = _lib.load()
    p = ctypes.c_void_p(1 << 20)
    q = ctypes.c_void_p(1 << 21)
    assert lib.cb_bilinear(0, 0, p, q, p, 4, 5, 0, 0, NULL) == 1


def test_empty_batch_is_noop():
    assert _lib.load().cb_bilinear(0, 0, NULL, NULL, NULL, 0, 8, 0, 0, NULL) == 0


def test_backward_output_aliasing_rejected_on_every_path():
    """cb_bilinear_bwd writes grad_a before the grad_b sum reads a: an output
    that aliases a, b, g or the other output is refused for every product and
    metric (not only on the Cl(8,0) matrix route)."""
    lib = _lib.load()
    a, b, g, o = (ctypes.c_void_p(k << 24) for k in range(1, 5))
    for op, n, neg in ((0, 8, 0), (0, 7, 1 << 6), (3, 9, 0), (5, 6, 0)):
        assert lib.cb_bilinear_bwd(op, a, b, g, a, o, 4, n, neg, 0, NULL) == 1
        assert lib.cb_bilinear_bwd(op, a, b, g, o, b, 4, n, neg, 0, NULL) == 1
        assert lib.cb_bilinear_bwd(op, a, b, g, g, o, 4, n, neg, 0, NULL) == 1
        assert lib.cb_bilinear_bwd(op, a, b, g, o, o, 4, n, neg, 0, NULL) == 1
        assert b"alias" in lib.cb_last_error() or b"different" in lib.cb_last_error()


def test_blade_map_arguments_rejected():
    lib = _lib.load()
    p = ctypes.c_void_p(1 << 20)
    q = ctypes.c_void_p(1 << 21)
    assert lib.cb_blade_map(9, p, q, 4, 5, 0, 0, 0, NULL) == 1      # kind out of range
    assert lib.cb_blade_map(3, p, q, 4, 5, 0, 0, 6, NULL) == 1      # grade > n
    assert lib.cb_blade_map(4, p, q, 4, 5, 0, 1, 0, NULL) == 1      # dual, degenerate
    assert b"degenerate" in lib.cb_last_error()
    assert lib.cb_blade_map(4, p, p, 4, 5, 0, 0, 0, NULL) == 1      # dual in place
    assert lib.cb_blade_map(0, NULL, NULL, 4, 5, 0, 0, 0, NULL) == 1  # null
    assert lib.cb_blade_map(0, NULL, NULL, 0, 5, 0, 0, 0, NULL) == 0  # empty batch
    assert lib.cb_norm_sq(p, q, 4, 0, 0, 0, NULL) == 3               # n = 0
    assert lib.cb_norm_sq(p, q, 4, 5, 1, 1, NULL) == 1               # both masks

