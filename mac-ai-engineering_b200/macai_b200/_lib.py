"""ctypes binding of the C ABI (include/gated_delta_b200.h) in libgated_delta_b200.so.

The library is built in-tree (macai_b200.build). There is no fallback: if it is missing or the device is not a B200,
every call raises.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

GD_OK, GD_ERR_ARG, GD_ERR_SHAPE, GD_ERR_ALIGN, GD_ERR_WORKSPACE, GD_ERR_LAUNCH, GD_ERR_TIMEOUT, GD_ERR_DEVICE = range(8)
GD_ERR_SCRATCH = 8
GD_FLOAT32, GD_FLOAT16, GD_BFLOAT16 = 0, 1, 2
GD_L2NORM, GD_STORE_STATES, GD_SCALE_Q, GD_STATES_STORED = 1, 2, 4, 8
GD_KEY_WIDTH_MASK = 0x00FF0000


def GD_KEY_WIDTH(dk: int) -> int:
    """Flags bits carrying the caller's key head width when q / k are zero-padded to 128 (the query scale's width)."""
    return (dk & 0xFF) << 16


GD_WIDE_STATE_PASS = 16  # gd_fwd_state: always two CTAs per (head, row) (the default picks four when they fit)
GD_TEST_WAIT_EXPIRES = 0x40000000  # test only: gd_fwd_state's first wait expires (the failure path's tests)

# every entry point declared in include/gated_delta_b200.h
EXPORTS = ("gd_status_string", "gd_workspace_bytes", "gd_prep", "gd_fwd_state", "gd_bwd_state", "gd_bwd_chunk",
           "gd_forward", "gd_backward", "gd_read_error", "gd_forward_noalloc", "gd_gates_fwd",
           "gd_gates_workspace_bytes", "gd_gates_bwd", "gd_gnorm_fwd", "gd_gnorm_workspace_bytes", "gd_gnorm_bwd",
           "gd_conv_fwd", "gd_conv_workspace_bytes", "gd_conv_bwd", "gd_workspace_bytes_packed", "gd_forward_packed",
           "gd_backward_packed")

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_DIMS = [_I] * 7 + [_I]          # dtype?, B, T, H, HK, DK, DV, flags (see each signature)
_SIGS = {
    "gd_status_string": ([_I], ctypes.c_char_p),
    "gd_workspace_bytes": ([_I, _I, _I, _I, _I, _I, _I], _SZ),
    "gd_prep": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "gd_fwd_state": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "gd_bwd_state": ([_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P], _I),
    "gd_bwd_chunk": ([_P] * 10 + [_I] * 8 + [_P, _SZ, _P], _I),
    "gd_forward": ([_P] * 8 + [_I] * 8 + [_P, _SZ, _P], _I),
    "gd_backward": ([_P] * 14 + [_I] * 8 + [_P, _SZ, _P], _I),
    "gd_read_error": ([_P, _P, ctypes.POINTER(_I)], _I),
    "gd_forward_noalloc": ([_P] * 8 + [_I] * 8 + [_P, ctypes.POINTER(_I)], _I),
    "gd_gates_fwd": ([_P] * 6 + [_I, _I, ctypes.c_longlong, _I, _P], _I),
    "gd_gates_workspace_bytes": ([ctypes.c_longlong, _I], _SZ),
    "gd_gates_bwd": ([_P] * 10 + [_I, _I, ctypes.c_longlong, _I, _P, _SZ, _P], _I),
    "gd_gnorm_fwd": ([_P] * 4 + [_I, _I, ctypes.c_longlong, _I, ctypes.c_float, _P], _I),
    "gd_gnorm_workspace_bytes": ([ctypes.c_longlong, _I], _SZ),
    "gd_gnorm_bwd": ([_P] * 7 + [_I, _I, ctypes.c_longlong, _I, ctypes.c_float, _P, _SZ, _P], _I),
    "gd_conv_fwd": ([_P] * 5 + [_I] * 9 + [_P], _I),
    "gd_conv_workspace_bytes": ([_I, _I, _I], _SZ),
    "gd_conv_bwd": ([_P] * 7 + [_I] * 9 + [_P, _SZ, _P], _I),
    "gd_workspace_bytes_packed": ([_I] * 7, _SZ),
    "gd_forward_packed": ([_P] * 9 + [_I] * 8 + [_P, _SZ, _P], _I),
    "gd_backward_packed": ([_P] * 15 + [_I] * 8 + [_P, _SZ, _P], _I),
}

_lib = None


class GatedDeltaError(RuntimeError):
    """A C-ABI call returned a failure status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = False):
    """The loaded library (ctypes.CDLL). Raises if it is not built (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path()):
        if not build_if_missing:
            raise RuntimeError(f"{path()} is not built: run `python -m macai_b200.build` (needs nvcc) first")
        _build.build()
    lib = ctypes.CDLL(path())
    for name, (args, res) in _SIGS.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    _lib = lib
    return lib


def status_string(status: int) -> str:
    try:
        return load().gd_status_string(status).decode()
    except Exception:  # the library itself is what failed
        return "unknown"


def check(status: int, what: str) -> None:
    if status != GD_OK:
        raise GatedDeltaError(status, what)
