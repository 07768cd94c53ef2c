"""The linear-attention layer's convolution path on B200, one CUDA pass each way (C ABI gd_conv_fwd / gd_conv_bwd in
libgated_delta_b200.so), mirroring the reference's src/macai/layer/_conv.py (`supported` :178-185, `ConvQKV`
:188-237, `conv_qkv` :240-241): the depthwise causal convolution (kernel 4, no bias) and its SiLU over the input
projection's [B, T, C] output, written directly as the rule's inputs:

    u[t, c] = sum_j w[c, j] x[t - 3 + j, c]       (zero before the sequence start; float32)
    y = u * sigmoid(u)                            (on the float32 u, one rounding)
    q, k = y's first two key_dim blocks as [B, T, H_v, D_k] in x's dtype, each key head written once for each of the
           `rep` value heads it serves (the repeat_interleave, without the copy)
    v    = the last value_dim channels as [B, T, H_v, D_v] in float32

The backward recomputes u from the saved x and returns dx [B, T, C] in x's dtype and, when the weight trains, dw in
its dtype and shape, summed in a fixed order (the same bits every run). There is no CPU path: CUDA tensors only.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

K = 4
_DTYPES = {torch.float32: _lib.GD_FLOAT32, torch.float16: _lib.GD_FLOAT16, torch.bfloat16: _lib.GD_BFLOAT16}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous with a 16-byte aligned start (a copy only when the view is not)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def supported(x, w, kd: int, dk: int, rep: int, dv: int) -> bool:
    """The cases the kernels take (the reference's supported(), _conv.py:178-185, with 16-byte channel groups):
    x [B, T, C] CUDA, C = 2 kd + vd, w with C * 4 elements in x's dtype or float32, kd a multiple of dk, vd of dv,
    (kd / dk) rep == vd / dv value heads, and C, kd, dk, dv multiples of 8 (16-bit x) or 4 (float32 x)."""
    if not (isinstance(x, torch.Tensor) and isinstance(w, torch.Tensor) and x.is_cuda and w.is_cuda):
        return False
    if x.dim() != 3 or x.dtype not in _DTYPES or w.dtype not in (x.dtype, torch.float32):
        return False
    C = x.shape[-1]
    vd = C - 2 * kd
    g = 4 if x.dtype == torch.float32 else 8
    return (w.numel() == C * K and w.shape[-1] == K and min(kd, dk, rep, dv) > 0 and vd > 0 and kd % dk == 0
            and vd % dv == 0 and (kd // dk) * rep == vd // dv and C % g == 0 and kd % g == 0 and dk % g == 0
            and dv % g == 0)


@torch.library.custom_op("macai_b200::conv_fwd", mutates_args=(), device_types="cuda")
def conv_fwd(x: torch.Tensor, w: torch.Tensor, kd: int, dk: int, rep: int,
             dv: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q, k, v): q, k [B, T, H_v, dk] in x's dtype, v [B, T, H_v, dv] float32; w is [C, 4]."""
    lib = _lib.load()
    B, T, C = x.shape
    hv = kd // dk * rep
    q = torch.empty((B, T, hv, dk), dtype=x.dtype, device=x.device)
    k = torch.empty((B, T, hv, dk), dtype=x.dtype, device=x.device)
    v = torch.empty((B, T, hv, dv), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        st = lib.gd_conv_fwd(_p(x), _p(w), _p(q), _p(k), _p(v), _DTYPES[x.dtype], _DTYPES[w.dtype], B, T, C, kd, dk,
                             rep, dv, _stream(x.device))
    _lib.check(st, "gd_conv_fwd")
    return q, k, v


@conv_fwd.register_fake
def _(x, w, kd, dk, rep, dv):
    B, T, C = x.shape
    hv = kd // dk * rep
    return (x.new_empty((B, T, hv, dk)), x.new_empty((B, T, hv, dk)),
            x.new_empty((B, T, hv, dv), dtype=torch.float32))


@torch.library.custom_op("macai_b200::conv_bwd", mutates_args=(), device_types="cuda")
def conv_bwd(x: torch.Tensor, w: torch.Tensor, dq: Optional[torch.Tensor], dk_: Optional[torch.Tensor],
             dv_: Optional[torch.Tensor], kd: int, dk: int, rep: int, dv: int,
             need_dw: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(dx, dw): dx like x, dw [C, 4] in w's dtype (an empty tensor unless asked for); a None cotangent is zero."""
    lib = _lib.load()
    dev = x.device
    B, T, C = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty((C, K), dtype=w.dtype, device=dev) if need_dw else w.new_empty(0)
    ws, nbytes = None, 0
    if need_dw:
        nbytes = lib.gd_conv_workspace_bytes(B, T, C)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_conv_bwd(_p(x), _p(w), _p(dq), _p(dk_), _p(dv_), _p(dx), _p(dw) if need_dw else None,
                             _DTYPES[x.dtype], _DTYPES[w.dtype], B, T, C, kd, dk, rep, dv, _p(ws), nbytes,
                             _stream(dev))
    _lib.check(st, "gd_conv_bwd")
    return dx, dw


@conv_bwd.register_fake
def _(x, w, dq, dk_, dv_, kd, dk, rep, dv, need_dw):
    return torch.empty_like(x), w.new_empty((x.shape[-1], K) if need_dw else (0,))


def _setup_context(ctx, inputs, output):
    x, w, kd, dk, rep, dv = inputs
    ctx.save_for_backward(x, w)
    ctx.dims = (kd, dk, rep, dv)


def _backward(ctx, dq, dk_, dv_):
    x, w = ctx.saved_tensors
    kd, dk, rep, dv = ctx.dims
    need_dw = bool(ctx.needs_input_grad[1])
    dq = None if dq is None else _aligned(dq.to(x.dtype))
    dk_ = None if dk_ is None else _aligned(dk_.to(x.dtype))
    dv_ = None if dv_ is None else _aligned(dv_.to(torch.float32))
    dx, dw = conv_bwd(x, w, dq, dk_, dv_, kd, dk, rep, dv, need_dw)
    return (dx if ctx.needs_input_grad[0] else None), (dw if need_dw else None), None, None, None, None


conv_fwd.register_autograd(_backward, setup_context=_setup_context)


class ConvQKV:
    """(q, k, v) = the convolution path of x [B, T, C]: `ConvQKV.apply(x, weight, kd, dk, rep, dv)`, the reference's
    autograd function (_conv.py:188-237). `weight` is the layer's conv1d weight ([C, 1, 4] or [C, 4])."""

    @staticmethod
    def apply(x, weight, kd, dk, rep, dv):
        if not supported(x, weight, kd, dk, rep, dv):
            raise ValueError("conv_qkv: x must be a CUDA [B, T, C] tensor with C = 2 kd + vd and the head widths "
                             "dividing it (multiples of 8 channels at 16 bits, 4 at float32); weight C x 4 in x's "
                             "dtype or float32")
        C = x.shape[-1]
        w = weight.reshape(C, K)
        q, k, v = conv_fwd(_aligned(x), _aligned(w), int(kd), int(dk), int(rep), int(dv))
        return q, k, v


def conv_qkv(x: torch.Tensor, weight: torch.Tensor, kd: int, dk: int, rep: int, dv: int):
    """q, k, v for the rule (the reference's conv_qkv(), _conv.py:240-241)."""
    return ConvQKV.apply(x, weight, kd, dk, rep, dv)
