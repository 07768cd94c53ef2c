"""The linear-attention layer's gates on B200, one CUDA pass each way (C ABI gd_gates_fwd / gd_gates_bwd in
libgated_delta_b200.so), mirroring the reference's src/macai/layer/_gates.py (`supported` :75-77, `Gates` :82-117,
`gates` :120-121):

    beta = sigmoid(b)                                   (float32)
    g    = -exp(A_log) * softplus(a + dt_bias)          (float32; softplus with PyTorch's threshold of 20)

from the [B, T, H_v] outputs of in_proj_b and in_proj_a; both results feed chunk_gated_delta_rule as float32. The
backward returns db, da in the inputs' dtype, and dA_log, dt_bias's gradient (in their dtype) only when they need one,
as per-head sums in a fixed order (the same bits every run). There is no CPU path: CUDA tensors only.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GD_FLOAT32, torch.float16: _lib.GD_FLOAT16, torch.bfloat16: _lib.GD_BFLOAT16}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def supported(b, a, A_log, dt_bias) -> bool:
    """The cases the kernels take (the reference's supported(), _gates.py:75-77): b and a of one float dtype and
    shape [..., H]; A_log and dt_bias [H] of one float dtype; CUDA tensors; fewer than 2^31 elements."""
    return (all(isinstance(t, torch.Tensor) and t.is_cuda for t in (b, a, A_log, dt_bias))
            and b.dtype in _DTYPES and A_log.dtype in _DTYPES and b.dtype == a.dtype and b.shape == a.shape
            and A_log.dtype == dt_bias.dtype and A_log.dim() == 1 and dt_bias.shape == A_log.shape
            and b.dim() >= 1 and b.shape[-1] == A_log.shape[0] and b.numel() < 2 ** 31)


@torch.library.custom_op("macai_b200::gates_fwd", mutates_args=(), device_types="cuda")
def gates_fwd(b: torch.Tensor, a: torch.Tensor, A_log: torch.Tensor,
              dt_bias: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(beta, g), both float32 with b's shape."""
    lib = _lib.load()
    dev = b.device
    beta = torch.empty(b.shape, dtype=torch.float32, device=dev)
    g = torch.empty(b.shape, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_gates_fwd(_p(b), _p(a), _p(A_log), _p(dt_bias), _p(beta), _p(g), _DTYPES[b.dtype],
                              _DTYPES[A_log.dtype], b.numel(), A_log.shape[0], _stream(dev))
    _lib.check(st, "gd_gates_fwd")
    return beta, g


@gates_fwd.register_fake
def _(b, a, A_log, dt_bias):
    return b.new_empty(b.shape, dtype=torch.float32), b.new_empty(b.shape, dtype=torch.float32)


@torch.library.custom_op("macai_b200::gates_bwd", mutates_args=(), device_types="cuda")
def gates_bwd(b: torch.Tensor, a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
              dbeta: Optional[torch.Tensor], dg: Optional[torch.Tensor], need_dA: bool,
              need_ddt: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(db, da, dA_log, ddt_bias); the last two are empty tensors unless asked for."""
    lib = _lib.load()
    dev = b.device
    H = A_log.shape[0]
    db, da = torch.empty_like(b), torch.empty_like(a)
    dA = torch.empty(H, dtype=A_log.dtype, device=dev) if need_dA else A_log.new_empty(0)
    ddt = torch.empty(H, dtype=dt_bias.dtype, device=dev) if need_ddt else dt_bias.new_empty(0)
    ws, nbytes = None, 0
    if need_dA or need_ddt:
        nbytes = lib.gd_gates_workspace_bytes(b.numel(), H)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_gates_bwd(_p(b), _p(a), _p(A_log), _p(dt_bias), _p(dbeta), _p(dg), _p(db), _p(da),
                              _p(dA) if need_dA else None, _p(ddt) if need_ddt else None, _DTYPES[b.dtype],
                              _DTYPES[A_log.dtype], b.numel(), H, _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_gates_bwd")
    return db, da, dA, ddt


@gates_bwd.register_fake
def _(b, a, A_log, dt_bias, dbeta, dg, need_dA, need_ddt):
    H = A_log.shape[0]
    return (torch.empty_like(b), torch.empty_like(a), A_log.new_empty(H if need_dA else 0),
            dt_bias.new_empty(H if need_ddt else 0))


def _setup_context(ctx, inputs, output):
    b, a, A_log, dt_bias = inputs
    ctx.save_for_backward(b, a, A_log, dt_bias)


def _backward(ctx, dbeta, dg):
    b, a, A_log, dt_bias = ctx.saved_tensors
    need_dA, need_ddt = bool(ctx.needs_input_grad[2]), bool(ctx.needs_input_grad[3])
    dbeta = None if dbeta is None else dbeta.float().contiguous()
    dg = None if dg is None else dg.float().contiguous()
    db, da, dA, ddt = gates_bwd(b, a, A_log, dt_bias, dbeta, dg, need_dA, need_ddt)
    return db, da, (dA if need_dA else None), (ddt if need_ddt else None)


gates_fwd.register_autograd(_backward, setup_context=_setup_context)


class Gates:
    """(beta, g) = (sigmoid(b), -exp(A_log) softplus(a + dt_bias)), both float32: `Gates.apply(b, a, A_log, dt_bias)`,
    the reference's autograd function (_gates.py:82-117)."""

    @staticmethod
    def apply(b, a, A_log, dt_bias):
        if not supported(b, a, A_log, dt_bias):
            raise ValueError("gates: b and a must be CUDA tensors of one float dtype and shape [..., H]; A_log and "
                             "dt_bias [H] of one float dtype")
        return gates_fwd(b.contiguous(), a.contiguous(), A_log.contiguous(), dt_bias.contiguous())


def gates(b: torch.Tensor, a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """beta, g for the rule (the reference's gates(), _gates.py:120-121)."""
    return Gates.apply(b, a, A_log, dt_bias)
