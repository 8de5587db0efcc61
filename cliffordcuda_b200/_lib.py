"""Loader for the native library ``libcliffordcuda_b200.so`` (C ABI, sm_100a).

The library is built in-tree (``python -m cliffordcuda_b200.build`` or
``__graft_entry__.build()``) and loaded with ctypes. There is no fallback: if
the library is missing or fails to load, every product raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcliffordcuda_b200.so")

# Mirrors include/cliffordcuda_b200.h
CB_OK = 0
STATUS_NAMES = {1: "CB_ERR_INVALID", 2: "CB_ERR_CUDA", 3: "CB_ERR_UNSUPPORTED",
                4: "CB_ERR_DEVICE"}
OPS = {"gp": 0, "wedge": 1, "inner": 2, "lc": 3, "rc": 4, "reg": 5}
MODES = {"fwd": 0, "grad_a": 1, "grad_b": 2}
MAPS = {"reverse": 0, "involute": 1, "conjugate": 2, "grade": 3, "dual": 4, "dual_t": 5}

# Every symbol include/cliffordcuda_b200.h declares, with its ctypes signature.
_i64, _i32, _u32, _vp = ctypes.c_int64, ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p
_f32 = ctypes.c_float
SIGNATURES = {
    "cb_bilinear": (_i32, [_i32, _i32, _vp, _vp, _vp, _i64, _i32, _u32, _u32, _vp]),
    "cb_bilinear_direct": (_i32, [_i32, _i32, _vp, _vp, _vp, _i64, _i32, _u32, _u32, _vp]),
    "cb_bilinear_bwd": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _u32, _u32, _vp]),
    "cb_layer_workspace_bytes": (_i32, [_i32, _i64, ctypes.POINTER(_i64)]),
    "cb_layer_prepare": (_i32, [_i32, _vp, _i32, _u32, _u32, _vp, _vp, _i64, _vp]),
    "cb_layer_forward": (_i32, [_vp, _vp, _vp, _i64, _i32, _vp]),
    "cb_layer_backward": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _i64, _i32, _u32, _u32, _vp,
                                 _i64, _vp]),
    "cb_layer_gp8_prepare": (_i32, [_vp, _vp, _vp]),
    "cb_layer_gp8_forward": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "cb_layer_gp8_backward": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp]),
    "cb_rotor_sizes": (_i32, [_i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "cb_rotor_compile": (_i32, [_vp, _i32, _vp, _vp, _vp]),
    "cb_rotor_apply": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "cb_rotor_workspace_bytes": (_i32, [_i32, _i64, ctypes.POINTER(_i64)]),
    "cb_rotor_apply_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _vp, _i64, _vp]),
    "cb_rotor_compile_bwd": (_i32, [_vp, _vp, _i32, _vp, _vp]),
    "cb_rotor_apply_bwd_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _vp]),
    "cb_blade_map": (_i32, [_i32, _vp, _vp, _i64, _i32, _u32, _u32, _i32, _vp]),
    "cb_norm_sq": (_i32, [_vp, _vp, _i64, _i32, _u32, _u32, _vp]),
    "cb_norm_sq_bwd": (_i32, [_vp, _vp, _vp, _i64, _i32, _u32, _u32, _vp]),
    "cb_last_error": (ctypes.c_char_p, []),
    "cb_device_status": (_i32, [_vp]),
    "cb_selftest_bounded_wait": (_i32, [_u32, _vp]),
    "cb_version": (_i32, []),
}

_lib = None
_lock = threading.Lock()


class CliffordNativeError(RuntimeError):
    """A native entry point returned an error status."""


def load():
    """Load the native library (once). Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"cliffordcuda_b200 native library not built: {LIB_PATH} is missing "
                    "(run `python -m cliffordcuda_b200.build`)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status, what):
    if status != CB_OK:
        msg = load().cb_last_error().decode(errors="replace")
        raise CliffordNativeError(f"{what} failed: {STATUS_NAMES.get(status, status)}: {msg}")


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def device_status(device=None):
    """Synchronise the current stream and raise if one of this library's
    kernels recorded a device-side failure (a bounded wait that expired)."""
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        check(load().cb_device_status(s), "cb_device_status")
