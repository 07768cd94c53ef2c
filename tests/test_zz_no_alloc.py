"""gd_forward_noalloc, the forward for callers that cannot allocate device memory, against gd_forward.

Some callers of this library cannot call cudaMalloc: their device memory all belongs to another allocator (a serving
engine's reserved pool, a host framework that owns the GPU), or cudaMalloc / cudaFree, which can synchronise the
device, are not allowed where they run. gd_forward_noalloc takes the same inputs and outputs as gd_forward but keeps
its intermediates in one fixed 64 MiB device array inside the library. These tests call both entry points through the
C ABI on the same inputs and require identical results (the same kernels on the same inputs, so the tolerance is
zero), on two calls in a row of different sizes, so that the second call also shows that what the first left in the
shared array does not leak into it; and they check that sizes beyond the array, and the stored-states flag (whose
workspace must outlive the call), are refused before any device call.

The file name makes pytest collect it last."""
import ctypes
import math

import pytest
import torch

from macai_b200 import _lib

pytestmark = pytest.mark.gpu

FLAGS = _lib.GD_L2NORM | _lib.GD_SCALE_Q


def make_inputs(B, T, H, HK, seed, D=128):
    """q, k, v ~ N(0, 1) in bf16; beta = sigmoid(N(0, 1)); g = -exp(U(0, log 16)) * softplus(N(0, 1)); s0 small."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HK, D, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, T, HK, D, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, T, H, D, generator=gen).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    g = -torch.exp(torch.rand(B, T, H, generator=gen) * math.log(16.0)) * torch.nn.functional.softplus(
        torch.randn(B, T, H, generator=gen))
    s0 = torch.randn(B, H, D, D, generator=gen) * 0.02
    return [x.cuda().contiguous() for x in (q, k, v, g, beta, s0)]


def forward(noalloc, q, k, v, g, beta, s0):
    lib = _lib.load()
    B, T, HK, D = q.shape
    H = v.shape[2]
    o = torch.empty_like(v)
    sT = torch.empty(B, H, D, D, device="cuda", dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    ptrs = [x.data_ptr() for x in (q, k, v, g, beta, s0, o, sT)]
    dims = [_lib.GD_BFLOAT16, B, T, H, HK, D, D, FLAGS]
    if noalloc:
        device_status = ctypes.c_int(-1)
        _lib.check(lib.gd_forward_noalloc(*ptrs, *dims, stream, ctypes.byref(device_status)), "gd_forward_noalloc")
        assert device_status.value == _lib.GD_OK, _lib.status_string(device_status.value)
    else:
        ws = torch.empty(lib.gd_workspace_bytes(B, T, H, HK, D, D, 0), dtype=torch.uint8, device="cuda")
        _lib.check(lib.gd_forward(*ptrs, *dims, ws.data_ptr(), ws.numel(), stream), "gd_forward")
        assert lib.gd_read_error(ws.data_ptr(), stream, None) == _lib.GD_OK
    torch.cuda.synchronize()
    return o, sT


def test_noalloc_matches_gd_forward_on_two_calls_in_a_row():
    for B, T, H, HK, seed in ((2, 300, 4, 2, 11), (1, 1000, 3, 3, 12)):
        x = make_inputs(B, T, H, HK, seed)
        o_ref, s_ref = forward(False, *x)
        o, s = forward(True, *x)
        assert torch.isfinite(o.float()).all() and torch.isfinite(s).all()
        assert torch.equal(o, o_ref), (B, T, H, HK, (o.float() - o_ref.float()).abs().max().item())
        assert torch.equal(s, s_ref), (B, T, H, HK, (s - s_ref).abs().max().item())


def test_noalloc_refuses_sizes_beyond_its_array_before_any_device_call():
    lib = _lib.load()
    # 16 value heads x 4,096 tokens need ~120 MiB of workspace; null pointers: nothing may be touched
    assert lib.gd_workspace_bytes(1, 4096, 16, 16, 128, 128, 0) > 64 << 20
    status = lib.gd_forward_noalloc(None, None, None, None, None, None, None, None, _lib.GD_BFLOAT16, 1, 4096, 16,
                                    16, 128, 128, FLAGS, None, None)
    assert status == _lib.GD_ERR_SCRATCH
    assert "64 MiB" in _lib.status_string(status)
    # the stored-states forward (its workspace must outlive the call) is refused up front
    status = lib.gd_forward_noalloc(None, None, None, None, None, None, None, None, _lib.GD_BFLOAT16, 1, 64, 1, 1,
                                    128, 128, FLAGS | _lib.GD_STORE_STATES, None, None)
    assert status == _lib.GD_ERR_ARG
