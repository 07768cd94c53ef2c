"""The gated RMSNorm on the rule's output on B200, one CUDA pass each way (C ABI gd_gnorm_fwd / gd_gnorm_bwd in
libgated_delta_b200.so), mirroring the reference's src/macai/layer/_gated_norm.py (`supported` :148-151,
`GatedRMSNorm` :154-197, `gated_rms_norm` :200-201) and transformers' Qwen3_5RMSNormGated with its rounding points:

    x_hat = x * rsqrt(mean(x^2) + eps)        (float32)
    h     = w * x_hat.to(x.dtype)              (rounded to x's dtype again when w has x's dtype)
    o     = (h * silu(z.float())).to(x.dtype)

The backward is float32 with one rounding per gradient; dw (in w's dtype) only when the weight needs a gradient, as a
sum over rows taken in a fixed order (the same bits every run). There is no CPU path: CUDA tensors only.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.GD_FLOAT32, torch.float16: _lib.GD_FLOAT16, torch.bfloat16: _lib.GD_BFLOAT16}
MAX_D = 1024


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous with a 16-byte aligned start (a copy only when the view is not)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def supported(x, z, w) -> bool:
    """The cases the kernels take (the reference's supported(), _gated_norm.py:148-151): x and z of one float dtype and
    shape [..., D]; w [D] in x's dtype or float32; D % 4 == 0 and 0 < D <= 1024; CUDA tensors."""
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in (x, z, w)) or x.dim() == 0:
        return False
    d = x.shape[-1]
    return (x.dtype in _DTYPES and x.dtype == z.dtype and x.shape == z.shape and w.dim() == 1 and w.shape[0] == d
            and d % 4 == 0 and 0 < d <= MAX_D and (w.dtype == x.dtype or w.dtype == torch.float32))


@torch.library.custom_op("macai_b200::gnorm_fwd", mutates_args=(), device_types="cuda")
def gnorm_fwd(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """o in x's dtype and shape."""
    lib = _lib.load()
    d = x.shape[-1]
    o = torch.empty_like(x)
    with torch.cuda.device(x.device):
        st = lib.gd_gnorm_fwd(_p(x), _p(z), _p(w), _p(o), _DTYPES[x.dtype], _DTYPES[w.dtype], x.numel() // d, d,
                              float(eps), _stream(x.device))
    _lib.check(st, "gd_gnorm_fwd")
    return o


@gnorm_fwd.register_fake
def _(x, z, w, eps):
    return torch.empty_like(x)


@torch.library.custom_op("macai_b200::gnorm_bwd", mutates_args=(), device_types="cuda")
def gnorm_bwd(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, do: torch.Tensor, eps: float,
              need_dw: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dx, dz, dw); dw is an empty tensor unless asked for."""
    lib = _lib.load()
    dev = x.device
    d = x.shape[-1]
    rows = x.numel() // d
    dx, dz = torch.empty_like(x), torch.empty_like(z)
    dw = torch.empty(d, dtype=w.dtype, device=dev) if need_dw else w.new_empty(0)
    ws, nbytes = None, 0
    if need_dw:
        nbytes = lib.gd_gnorm_workspace_bytes(rows, d)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_gnorm_bwd(_p(x), _p(z), _p(w), _p(do), _p(dx), _p(dz), _p(dw) if need_dw else None,
                              _DTYPES[x.dtype], _DTYPES[w.dtype], rows, d, float(eps), _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_gnorm_bwd")
    return dx, dz, dw


@gnorm_bwd.register_fake
def _(x, z, w, do, eps, need_dw):
    return torch.empty_like(x), torch.empty_like(z), w.new_empty(w.shape[0] if need_dw else 0)


def _setup_context(ctx, inputs, output):
    x, z, w, eps = inputs
    ctx.save_for_backward(x, z, w)
    ctx.eps = eps


def _backward(ctx, do):
    x, z, w = ctx.saved_tensors
    need_dw = bool(ctx.needs_input_grad[2])
    do = _aligned(do.to(x.dtype))
    dx, dz, dw = gnorm_bwd(x, z, w, do, ctx.eps, need_dw)
    return dx, dz, (dw if need_dw else None), None


gnorm_fwd.register_autograd(_backward, setup_context=_setup_context)


class GatedRMSNorm:
    """o = (w * rmsnorm(x).to(x.dtype)) * silu(z.float()), cast to x's dtype: `GatedRMSNorm.apply(x, z, w, eps)`, the
    reference's autograd function (_gated_norm.py:154-197)."""

    @staticmethod
    def apply(x, z, w, eps):
        if not supported(x, z, w):
            raise ValueError("gated_rms_norm: x and z must be CUDA tensors of one float dtype and shape [..., D] with "
                             "D % 4 == 0 and D <= 1024; w [D] in x's dtype or float32")
        return gnorm_fwd(_aligned(x), _aligned(z), _aligned(w), float(eps))


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The gated RMSNorm (the reference's gated_rms_norm(), _gated_norm.py:200-201)."""
    return GatedRMSNorm.apply(x, z, w, eps)
