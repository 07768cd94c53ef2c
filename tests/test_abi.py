"""The C ABI library without a GPU: it loads, exports every entry point include/gated_delta_b200.h declares, sizes
workspaces, and refuses bad arguments with status codes before touching a device (no compute calls here)."""
import ctypes
import os
import re

import pytest

from macai_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gated_delta_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const char\*|size_t|int)\s+(gd_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 9
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(_lib.EXPORTS) == names


def test_status_strings():
    lib = _lib.load()
    for s in range(8):
        assert lib.gd_status_string(s)
    assert b"unknown" in lib.gd_status_string(99)


def test_workspace_sizes():
    lib = _lib.load()
    f = lib.gd_workspace_bytes(4, 1024, 16, 16, 128, 128, 0)
    b = lib.gd_workspace_bytes(4, 1024, 16, 16, 128, 128, 1)
    assert 0 < f < b
    assert lib.gd_workspace_bytes(8, 1024, 16, 16, 128, 128, 1) > b          # grows with the batch
    assert lib.gd_workspace_bytes(4, 1000, 16, 16, 128, 128, 0) == f         # chunks of 64 tokens
    assert lib.gd_workspace_bytes(4, 1024, 16, 16, 64, 128, 1) == 0          # head width not built
    assert lib.gd_workspace_bytes(4, 1024, 15, 4, 128, 128, 1) == 0          # value heads not a multiple of key heads


def test_refusals_before_any_device_call():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(256)
    st = lib.gd_prep(one, one, one, one, one, _lib.GD_BFLOAT16, 1, 64, 1, 1, 96, 128, 0, one, 1 << 30, nul)
    assert st == _lib.GD_ERR_SHAPE
    st = lib.gd_prep(nul, one, one, one, one, _lib.GD_BFLOAT16, 1, 64, 1, 1, 128, 128, 0, one, 1 << 30, nul)
    assert st == _lib.GD_ERR_ARG
    st = lib.gd_prep(one, one, one, one, one, 7, 1, 64, 1, 1, 128, 128, 0, one, 1 << 30, nul)
    assert st == _lib.GD_ERR_ARG
    st = lib.gd_prep(ctypes.c_void_p(257), one, one, one, one, _lib.GD_BFLOAT16, 1, 64, 1, 1, 128, 128, 0, one,
                     1 << 30, nul)
    assert st == _lib.GD_ERR_ALIGN
    st = lib.gd_forward(one, one, one, one, one, nul, one, nul, _lib.GD_BFLOAT16, 0, 64, 1, 1, 128, 128, 0, one,
                        1 << 30, nul)
    assert st == _lib.GD_ERR_SHAPE


def test_error_type_carries_status():
    e = _lib.GatedDeltaError(_lib.GD_ERR_TIMEOUT, "gd_forward")
    assert e.status == _lib.GD_ERR_TIMEOUT and "gd_forward" in str(e)
    with pytest.raises(_lib.GatedDeltaError):
        _lib.check(_lib.GD_ERR_SHAPE, "x")


def test_gates_refusals_before_any_device_call():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(256)
    # n not a multiple of H, unknown dtype, null outputs: status codes, nothing launched
    assert lib.gd_gates_fwd(one, one, one, one, one, one, 2, 0, 100, 16, nul) == _lib.GD_ERR_SHAPE
    assert lib.gd_gates_fwd(one, one, one, one, one, one, 7, 0, 64, 16, nul) == _lib.GD_ERR_ARG
    assert lib.gd_gates_fwd(one, one, one, one, nul, one, 2, 0, 64, 16, nul) == _lib.GD_ERR_ARG
    assert lib.gd_gates_fwd(nul, nul, nul, nul, nul, nul, 2, 0, 0, 16, nul) == _lib.GD_OK  # no elements
    # per-head sums without a workspace
    ws = lib.gd_gates_workspace_bytes(64 * 1024, 16)
    assert ws >= 2 * 16 * 4 and lib.gd_gates_workspace_bytes(100, 16) == 0
    assert lib.gd_gates_bwd(one, one, one, one, one, one, one, one, one, nul, 2, 0, 64 * 1024, 16, nul, 0,
                            nul) == _lib.GD_ERR_WORKSPACE


def test_gated_norm_refusals_before_any_device_call():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(258)
    BF, F16, F32 = _lib.GD_BFLOAT16, _lib.GD_FLOAT16, _lib.GD_FLOAT32
    # widths: D % 4, D > 1024; weight dtype neither x's nor float32; unknown dtype; null and misaligned pointers
    assert lib.gd_gnorm_fwd(one, one, one, one, BF, BF, 10, 126, 1e-6, nul) == _lib.GD_ERR_SHAPE
    assert lib.gd_gnorm_fwd(one, one, one, one, BF, BF, 10, 2048, 1e-6, nul) == _lib.GD_ERR_SHAPE
    assert lib.gd_gnorm_fwd(one, one, one, one, BF, F16, 10, 128, 1e-6, nul) == _lib.GD_ERR_ARG
    assert lib.gd_gnorm_fwd(one, one, one, one, 9, F32, 10, 128, 1e-6, nul) == _lib.GD_ERR_ARG
    assert lib.gd_gnorm_fwd(one, one, one, nul, BF, F32, 10, 128, 1e-6, nul) == _lib.GD_ERR_ARG
    assert lib.gd_gnorm_fwd(one, odd, one, one, BF, F32, 10, 128, 1e-6, nul) == _lib.GD_ERR_ALIGN
    assert lib.gd_gnorm_fwd(nul, nul, nul, nul, BF, BF, 0, 128, 1e-6, nul) == _lib.GD_OK  # no rows
    # the weight's gradient without a workspace
    assert lib.gd_gnorm_workspace_bytes(65536, 128) >= 128 * 4 and lib.gd_gnorm_workspace_bytes(10, 0) == 0
    assert lib.gd_gnorm_bwd(one, one, one, one, one, one, one, BF, BF, 65536, 128, 1e-6, nul, 0,
                            nul) == _lib.GD_ERR_WORKSPACE


def test_conv_refusals_before_any_device_call():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(264)  # 8-byte aligned only
    BF, F16, F32 = _lib.GD_BFLOAT16, _lib.GD_FLOAT16, _lib.GD_FLOAT32
    # (B, T, C, KD, DK, REP, DV) of the 9B layer, then broken ones
    ok = (2, 33, 8192, 2048, 128, 2, 128)
    bad_shapes = [(2, 33, 8192, 2048, 128, 1, 128),   # value heads != key heads x rep
                  (2, 33, 8196, 2048, 128, 2, 128),   # VD not a multiple of DV
                  (2, 33, 4096, 2048, 128, 2, 128),   # no value channels
                  (2, 33, 8192, 2048, 100, 2, 128)]   # DK does not divide KD / not a multiple of 8
    for shp in bad_shapes:
        assert lib.gd_conv_fwd(one, one, one, one, one, BF, BF, *shp, nul) == _lib.GD_ERR_SHAPE, shp
    assert lib.gd_conv_fwd(one, one, one, one, one, BF, F16, *ok, nul) == _lib.GD_ERR_ARG
    assert lib.gd_conv_fwd(one, one, nul, one, one, BF, BF, *ok, nul) == _lib.GD_ERR_ARG
    assert lib.gd_conv_fwd(odd, one, one, one, one, BF, BF, *ok, nul) == _lib.GD_ERR_ALIGN
    assert lib.gd_conv_fwd(nul, nul, nul, nul, nul, BF, BF, 0, 33, 8192, 2048, 128, 2, 128, nul) == _lib.GD_OK
    assert lib.gd_conv_workspace_bytes(2, 33, 8192) >= 8192 * 4 * 4 and lib.gd_conv_workspace_bytes(2, 33, 0) == 0
    assert lib.gd_conv_bwd(one, one, one, one, one, one, one, BF, BF, *ok, nul, 0, nul) == _lib.GD_ERR_WORKSPACE


def test_packed_refusals_before_any_device_call():
    lib = _lib.load()
    nul = ctypes.c_void_p(0)
    one = ctypes.c_void_p(256)
    BF = _lib.GD_BFLOAT16
    # (N, dtype, T, H, HK, DK, DV, flags)
    assert lib.gd_workspace_bytes_packed(0, 100, 16, 16, 128, 128, 1) == 0          # no sequences
    assert lib.gd_workspace_bytes_packed(3, 100, 16, 16, 64, 128, 1) == 0           # head width
    n1 = lib.gd_workspace_bytes_packed(3, 100, 16, 16, 128, 128, 1)
    n0 = lib.gd_workspace_bytes_packed(3, 100, 16, 16, 128, 128, 0)
    assert n1 > n0 > 0
    # more sequences add chunks (each starts a new one): a larger workspace
    assert lib.gd_workspace_bytes_packed(50, 100, 16, 16, 128, 128, 0) > n0
    args = [one] * 8
    assert lib.gd_forward_packed(*args, nul, 3, BF, 100, 16, 16, 128, 128, 5, one, n0, nul) == _lib.GD_ERR_ARG
    assert lib.gd_forward_packed(*args, one, 0, BF, 100, 16, 16, 128, 128, 5, one, n0, nul) == _lib.GD_ERR_SHAPE
    assert lib.gd_forward_packed(*args, one, 3, BF, 100, 16, 16, 128, 128, 5, one, n0 - 256,
                                 nul) == _lib.GD_ERR_WORKSPACE
    grads = [one] * 14
    assert lib.gd_backward_packed(*grads, one, 3, BF, 100, 16, 16, 128, 128, 5, one, n0, nul) == _lib.GD_ERR_WORKSPACE
