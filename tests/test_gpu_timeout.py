"""The bounded-wait failure path on the GPU, in the allowed form: a wait on a barrier that nothing signals.

Every device wait of the kernels (an mbarrier) gives up after a clock budget, records GD_ERR_TIMEOUT and the stage in
the workspace's error word, and lets the kernel fall through to its clean-up. The test-only flag GD_TEST_WAIT_EXPIRES
makes gd_fwd_state's MMA-issuing thread wait ~1 ms on a barrier nobody arrives on before it issues anything; the other
roles of each CTA (16 epilogue warps, the stage loader with two stages of bulk copies in flight) then give up in their
own bounded waits, the loader lets its copies land, and the CTA frees its TMEM and returns. Checked: the launch
returns, gd_read_error reports (GD_ERR_TIMEOUT, stage 28) once and then GD_OK (the word is cleared), the context
stays usable, and a normal call on the same workspace afterwards gives the same bits as a call on a fresh one."""
import ctypes
import time

import pytest
import torch

from macai_b200 import _lib
from test_zz_no_alloc import make_inputs

pytestmark = pytest.mark.gpu
FLAGS = _lib.GD_L2NORM | _lib.GD_SCALE_Q


def _ptrs(*xs):
    return [None if x is None else ctypes.c_void_p(x.data_ptr()) for x in xs]


def _forward(lib, ws, x, stream):
    q, k, v, g, beta, s0 = x
    B, T, HK, D = q.shape
    H = v.shape[2]
    o = torch.empty_like(v)
    sT = torch.empty(B, H, D, D, device="cuda")
    _lib.check(lib.gd_forward(*_ptrs(q, k, v, g, beta, s0, o, sT), _lib.GD_BFLOAT16, B, T, H, HK, D, D, FLAGS,
                              ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "gd_forward")
    return o, sT


@pytest.mark.parametrize("store", [False, True])
def test_expired_wait_reports_timeout_and_next_call_is_exact(store):
    lib = _lib.load()
    x = make_inputs(2, 300, 2, 2, seed=21)   # 5 chunks per row: the loader has two stages in flight when it waits
    q, k, v, g, beta, s0 = x
    B, T, HK, D = q.shape
    H = v.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    nbytes = lib.gd_workspace_bytes(B, T, H, HK, D, D, 1)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    o = torch.empty_like(v)
    sT = torch.empty(B, H, D, D, device="cuda")
    _lib.check(lib.gd_prep(*_ptrs(q, k, v, g, beta), _lib.GD_BFLOAT16, B, T, H, HK, D, D, FLAGS,
                           ctypes.c_void_p(ws.data_ptr()), nbytes, stream), "gd_prep")
    flags = FLAGS | _lib.GD_TEST_WAIT_EXPIRES | (_lib.GD_STORE_STATES if store else 0)
    t0 = time.time()
    _lib.check(lib.gd_fwd_state(*_ptrs(s0, o, sT), _lib.GD_BFLOAT16, B, T, H, HK, D, D, flags,
                                ctypes.c_void_p(ws.data_ptr()), nbytes, stream), "gd_fwd_state")
    where = ctypes.c_int(-1)
    code = lib.gd_read_error(ctypes.c_void_p(ws.data_ptr()), stream, ctypes.byref(where))
    took = time.time() - t0
    assert code == _lib.GD_ERR_TIMEOUT, _lib.status_string(code)
    assert where.value == 28
    assert took < 30, took
    assert lib.gd_read_error(ctypes.c_void_p(ws.data_ptr()), stream, None) == _lib.GD_OK  # cleared
    torch.cuda.synchronize()                                                                 # context usable
    o1, s1 = _forward(lib, ws, x, stream)
    assert lib.gd_read_error(ctypes.c_void_p(ws.data_ptr()), stream, None) == _lib.GD_OK
    fresh = torch.empty_like(ws)
    o2, s2 = _forward(lib, fresh, x, stream)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
