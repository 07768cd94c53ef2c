"""The gated delta rule on B200: torch custom ops over the sm_100a kernels (libgated_delta_b200.so, C ABI in
include/gated_delta_b200.h), and the drop-in for transformers' torch_chunk_gated_delta_rule (same arguments, same
returns). Mirrors the reference's src/macai/gated_delta/op.py: `chunk_gated_delta_rule` (:264-298), the autograd
function `GatedDeltaRule` (:116-257), `l2norm` (:260-261) and `recurrent_reference` (:301-314).

There is no CPU or PyTorch fallback: on anything but a CUDA tensor on an sm_100 device the ops raise.
"""
from __future__ import annotations

import collections
import ctypes
import math
from typing import Optional

import torch

from .. import _lib

# The chunk length of every kernel (tokens). The drop-in accepts `chunk_size` for signature compatibility and, like the
# reference (op.py:268-269), runs its own chunking; 64 is also the value every caller passes.
CHUNK = 64
# Head widths the kernels are built for (the Qwen3.5 / Qwen3-Next linear-attention shapes); narrower multiples of 32
# are zero-padded to it by the drop-in (_pad_heads).
HEAD_DIMS = (128,)
# What each call ran, as the reference's op.CALLS (op.py:44-46): "fwd", "fwd stored", "bwd", "bwd stored".
CALLS: collections.Counter = collections.Counter()
# RECOMPUTE_STATES, as the reference's setting (op.py:27-33), read at each call: True (the default) = a training forward
# keeps only its inputs and the backward recomputes the chunk matrices, states and Vn; False = the training forward
# writes them into a workspace the autograd context keeps until the backward (gd_workspace_bytes(..., 1) of device
# memory per call), and the backward skips the recompute. Outputs and gradients are the same bits either way.
RECOMPUTE_STATES = True
# The kernels compute every product with bf16 tensor-core operands (fp32 accumulation; the operands whose rounding would
# break the bf16 parity bar are carried as bf16 hi + lo pairs). That meets the reference's bar for bf16 queries, not its
# float16 or float32 bars: measured against transformers' own error on the same inputs, fp16 queries come out 2-8x and
# fp32 queries 300-20,000x less accurate. So a float16 / float32 query is refused (NotImplementedError), as the
# reference refuses what it cannot compute exactly, unless ALLOW_BF16_COMPUTE is True: then such inputs run through the
# same kernels (read in their own dtype, results in the query's dtype) with bf16-grade accuracy. A bfloat16 query with
# a float32 value (the reference layer's convolution path writes v in fp32) is accepted: v is rounded to bf16, and the
# results meet the bf16 bar against transformers run on the same mixed inputs.
ALLOW_BF16_COMPUTE = False

_DTYPES = {torch.float32: _lib.GD_FLOAT32, torch.float16: _lib.GD_FLOAT16, torch.bfloat16: _lib.GD_BFLOAT16}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dims(q: torch.Tensor, v: torch.Tensor):
    B, T, HK, DK = q.shape
    H, DV = v.shape[2], v.shape[3]
    return B, T, H, HK, DK, DV


def check_dtype(dt) -> None:
    """The query dtypes the kernels serve at the reference's accuracy (bfloat16), or any of float16 / float32 /
    bfloat16 with ALLOW_BF16_COMPUTE; TypeError for other dtypes, NotImplementedError for the refused ones."""
    if dt not in _DTYPES:
        raise TypeError(f"query dtype {dt} is not supported (float32, float16, bfloat16)")
    if dt != torch.bfloat16 and not ALLOW_BF16_COMPUTE:
        raise NotImplementedError(
            f"{dt} queries: the B200 kernels compute with bf16 tensor-core operands, whose results miss the reference's "
            f"{dt} accuracy; pass bfloat16 inputs, or set macai_b200.gated_delta.op.ALLOW_BF16_COMPUTE = True to "
            "accept bf16-grade results in the input dtype")


def check_shapes(q, k, v, g, beta, s0=None) -> None:
    """The refusals the kernels need, raised before any launch (ValueError / NotImplementedError, as the reference's
    op.py:124-131 and _chunked.py:1228-1231)."""
    if q.dim() != 4 or k.shape != q.shape or v.dim() != 4:
        raise ValueError(f"query/key must be [B, T, H, DK] and value [B, T, H, DV]; got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    B, T, H, HK, DK, DV = _dims(q, v)
    if v.shape[:2] != q.shape[:2]:
        raise ValueError("query and value must share batch and sequence dimensions")
    if H % HK != 0:
        raise ValueError(f"value heads ({H}) must be a multiple of key heads ({HK})")
    if DK % 32 != 0 or DV % 32 != 0:
        raise ValueError(f"head widths must be multiples of 32 (the reference's op.py:124-125); got DK={DK}, DV={DV}")
    if DK > max(HEAD_DIMS) or DV > max(HEAD_DIMS):
        raise NotImplementedError(f"the B200 kernels are built for head widths up to {max(HEAD_DIMS)} (narrower heads "
                                  f"are zero-padded to it); got DK={DK}, DV={DV}")
    if g.shape != (B, T, H) or beta.shape != (B, T, H):
        raise ValueError(f"g and beta must be [B, T, H] = {(B, T, H)}; got {tuple(g.shape)}, {tuple(beta.shape)}")
    if s0 is not None and s0.shape != (B, H, DK, DV):
        raise ValueError(f"initial_state must be [B, H, DK, DV] = {(B, H, DK, DV)}; got {tuple(s0.shape)}")
    if q.device.type != "cuda":
        raise RuntimeError("macai_b200's gated delta rule runs on CUDA (B200) tensors only; there is no CPU path")


def workspace_bytes(B, T, H, HK, DK, DV, backward: bool) -> int:
    n = _lib.load().gd_workspace_bytes(B, T, H, HK, DK, DV, int(backward))
    if n == 0:
        raise NotImplementedError(f"unsupported sizes B={B} T={T} H={H} HK={HK} DK={DK} DV={DV}")
    return n


# ------------------------------------------------------------------------------------------------------------------
# custom ops

@torch.library.custom_op("macai_b200::gated_delta_fwd", mutates_args=(), device_types="cuda")
def gated_delta_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                    s0: Optional[torch.Tensor], flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    """o [B, T, H, DV] (q's dtype) and S_T [B, H, DK, DV] fp32. q, k [B, T, HK, DK]; v [B, T, H, DV] in q's dtype;
    g, beta fp32 [B, T, H]; s0 fp32 or None. flags: GD_L2NORM | GD_SCALE_Q (| GD_WIDE_STATE_PASS)."""
    B, T, H, HK, DK, DV = _dims(q, v)
    lib = _lib.load()
    dev = q.device
    o = torch.empty(B, T, H, DV, dtype=q.dtype, device=dev)
    sT = torch.empty(B, H, DK, DV, dtype=torch.float32, device=dev)
    nbytes = workspace_bytes(B, T, H, HK, DK, DV, False)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_forward(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(o), _p(sT), _DTYPES[q.dtype], B, T, H, HK,
                            DK, DV, flags, _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_forward")
    CALLS["fwd"] += 1
    return o, sT


@gated_delta_fwd.register_fake
def _(q, k, v, g, beta, s0, flags):
    B, T, H, HK, DK, DV = _dims(q, v)
    return q.new_empty(B, T, H, DV), q.new_empty(B, H, DK, DV, dtype=torch.float32)


@torch.library.custom_op("macai_b200::gated_delta_fwd_stored", mutates_args=(), device_types="cuda")
def gated_delta_fwd_stored(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           s0: Optional[torch.Tensor], flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The stored-states training forward (RECOMPUTE_STATES = False; the reference's op.py:141-155, :165-167): o and
    S_T as gated_delta_fwd, plus the workspace (uint8) holding every chunk matrix, state and Vn the backward reads."""
    B, T, H, HK, DK, DV = _dims(q, v)
    lib = _lib.load()
    dev = q.device
    o = torch.empty(B, T, H, DV, dtype=q.dtype, device=dev)
    sT = torch.empty(B, H, DK, DV, dtype=torch.float32, device=dev)
    nbytes = workspace_bytes(B, T, H, HK, DK, DV, True)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_forward(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(o), _p(sT), _DTYPES[q.dtype], B, T, H, HK,
                            DK, DV, flags | _lib.GD_STORE_STATES, _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_forward")
    CALLS["fwd stored"] += 1
    return o, sT, ws


@gated_delta_fwd_stored.register_fake
def _(q, k, v, g, beta, s0, flags):
    B, T, H, HK, DK, DV = _dims(q, v)
    nbytes = workspace_bytes(B, T, H, HK, DK, DV, True)
    return (q.new_empty(B, T, H, DV), q.new_empty(B, H, DK, DV, dtype=torch.float32),
            q.new_empty(nbytes, dtype=torch.uint8))


@torch.library.custom_op("macai_b200::gated_delta_bwd", mutates_args=(), device_types="cuda")
def gated_delta_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                    s0: Optional[torch.Tensor], do: torch.Tensor, dsT: Optional[torch.Tensor],
                    flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                         torch.Tensor]:
    """(dq, dk, dv, dg, dbeta, ds0): the chunk states recomputed from the inputs (the reference's recompute mode,
    op.py:207-218), then the reverse state pass and the per-chunk gradients."""
    B, T, H, HK, DK, DV = _dims(q, v)
    lib = _lib.load()
    dev = q.device
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(B, T, H, dtype=torch.float32, device=dev)
    dbeta = torch.empty(B, T, H, dtype=torch.float32, device=dev)
    ds0 = torch.empty(B, H, DK, DV, dtype=torch.float32, device=dev)
    nbytes = workspace_bytes(B, T, H, HK, DK, DV, True)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_backward(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(do), _p(dsT), _p(dq), _p(dk), _p(dv),
                             _p(dg), _p(dbeta), _p(ds0), _DTYPES[q.dtype], B, T, H, HK, DK, DV, flags, _p(ws), nbytes,
                             _stream(dev))
    _lib.check(st, "gd_backward")
    CALLS["bwd"] += 1
    return dq, dk, dv, dg, dbeta, ds0


@gated_delta_bwd.register_fake
def _(q, k, v, g, beta, s0, do, dsT, flags):
    B, T, H, HK, DK, DV = _dims(q, v)
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), q.new_empty(B, T, H, **f32),
            q.new_empty(B, T, H, **f32), q.new_empty(B, H, DK, DV, **f32))


# ws is declared unmutated: the backward rewrites only the workspace's backward scratch area (the reverse pass's dS,
# dVn and dO images and partial sums), which holds nothing between calls and is always written before it is read; the
# kept states are only read. (Declaring it mutated would bump the saved tensor's version and refuse a second
# backward over a retained graph.)
@torch.library.custom_op("macai_b200::gated_delta_bwd_stored", mutates_args=(), device_types="cuda")
def gated_delta_bwd_stored(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor, do: torch.Tensor,
                           dsT: Optional[torch.Tensor], ws: torch.Tensor,
                           flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                torch.Tensor]:
    """(dq, dk, dv, dg, dbeta, ds0) from the states gated_delta_fwd_stored kept in ws (the reference's stored mode,
    op.py:204-206): the reverse state pass and the per-chunk gradients only."""
    B, T, H, HK, DK, DV = _dims(q, v)
    lib = _lib.load()
    dev = q.device
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(B, T, H, dtype=torch.float32, device=dev)
    dbeta = torch.empty(B, T, H, dtype=torch.float32, device=dev)
    ds0 = torch.empty(B, H, DK, DV, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_backward(_p(q), _p(k), _p(v), None, _p(beta), None, _p(do), _p(dsT), _p(dq), _p(dk), _p(dv),
                             _p(dg), _p(dbeta), _p(ds0), _DTYPES[q.dtype], B, T, H, HK, DK, DV,
                             flags | _lib.GD_STATES_STORED, _p(ws), ws.numel(), _stream(dev))
    _lib.check(st, "gd_backward")
    CALLS["bwd stored"] += 1
    return dq, dk, dv, dg, dbeta, ds0


@gated_delta_bwd_stored.register_fake
def _(q, k, v, beta, do, dsT, ws, flags):
    B, T, H, HK, DK, DV = _dims(q, v)
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), q.new_empty(B, T, H, **f32),
            q.new_empty(B, T, H, **f32), q.new_empty(B, H, DK, DV, **f32))


def _setup_context(ctx, inputs, output):
    q, k, v, g, beta, s0, flags = inputs
    ctx.save_for_backward(q, k, v, g, beta, s0)
    ctx.flags = flags
    ctx.has_s0 = s0 is not None


def _backward(ctx, do, dsT):
    q, k, v, g, beta, s0 = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*v.shape, dtype=q.dtype, device=q.device)
    do = do.to(q.dtype).contiguous()
    dsT = None if dsT is None else dsT.to(torch.float32).contiguous()
    dq, dk, dv, dg, dbeta, ds0 = gated_delta_bwd(q, k, v, g, beta, s0, do, dsT, ctx.flags)
    return dq, dk, dv, dg, dbeta, (ds0 if ctx.has_s0 else None), None


gated_delta_fwd.register_autograd(_backward, setup_context=_setup_context)


def _setup_context_stored(ctx, inputs, output):
    q, k, v, g, beta, s0, flags = inputs
    ctx.save_for_backward(q, k, v, beta, output[2])
    ctx.flags = flags
    ctx.has_s0 = s0 is not None


def _backward_stored(ctx, do, dsT, _dws):
    q, k, v, beta, ws = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*v.shape, dtype=q.dtype, device=q.device)
    do = do.to(q.dtype).contiguous()
    dsT = None if dsT is None else dsT.to(torch.float32).contiguous()
    dq, dk, dv, dg, dbeta, ds0 = gated_delta_bwd_stored(q, k, v, beta, do, dsT, ws, ctx.flags)
    return dq, dk, dv, dg, dbeta, (ds0 if ctx.has_s0 else None), None


gated_delta_fwd_stored.register_autograd(_backward_stored, setup_context=_setup_context_stored)


# ------------------------------------------------------------------------------------------------------------------
# packed rows (cu_seqlens): q, k, v, g, beta carry one batch row of T tokens holding N sequences; s0 / S_T are
# [N, H, DK, DV]; every sequence runs as its own row (the C ABI's gd_forward_packed / gd_backward_packed)

def packed_workspace_bytes(N, T, H, HK, DK, DV, backward: bool) -> int:
    n = _lib.load().gd_workspace_bytes_packed(N, T, H, HK, DK, DV, int(backward))
    if n == 0:
        raise NotImplementedError(f"unsupported packed sizes N={N} T={T} H={H} HK={HK} DK={DK} DV={DV}")
    return n


def _pdims(q, v, cu):
    _, T, HK, DK = q.shape
    return cu.numel() - 1, T, v.shape[2], HK, DK, v.shape[3]


@torch.library.custom_op("macai_b200::gated_delta_fwd_packed", mutates_args=(), device_types="cuda")
def gated_delta_fwd_packed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           s0: Optional[torch.Tensor], cu: torch.Tensor,
                           flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    """o [1, T, H, DV] and S_T [N, H, DK, DV] over packed rows; cu: int32 [N + 1] on the device."""
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    lib = _lib.load()
    dev = q.device
    o = torch.empty(1, T, H, DV, dtype=q.dtype, device=dev)
    sT = torch.empty(N, H, DK, DV, dtype=torch.float32, device=dev)
    nbytes = packed_workspace_bytes(N, T, H, HK, DK, DV, False)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_forward_packed(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(o), _p(sT), _p(cu), N,
                                   _DTYPES[q.dtype], T, H, HK, DK, DV, flags, _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_forward_packed")
    CALLS["fwd packed"] += 1
    return o, sT


@gated_delta_fwd_packed.register_fake
def _(q, k, v, g, beta, s0, cu, flags):
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    return q.new_empty(1, T, H, DV), q.new_empty(N, H, DK, DV, dtype=torch.float32)


@torch.library.custom_op("macai_b200::gated_delta_fwd_packed_stored", mutates_args=(), device_types="cuda")
def gated_delta_fwd_packed_stored(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                                  beta: torch.Tensor, s0: Optional[torch.Tensor], cu: torch.Tensor,
                                  flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The stored-states training forward over packed rows: o, S_T and the workspace the backward reads."""
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    lib = _lib.load()
    dev = q.device
    o = torch.empty(1, T, H, DV, dtype=q.dtype, device=dev)
    sT = torch.empty(N, H, DK, DV, dtype=torch.float32, device=dev)
    nbytes = packed_workspace_bytes(N, T, H, HK, DK, DV, True)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_forward_packed(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(o), _p(sT), _p(cu), N,
                                   _DTYPES[q.dtype], T, H, HK, DK, DV, flags | _lib.GD_STORE_STATES, _p(ws), nbytes,
                                   _stream(dev))
    _lib.check(st, "gd_forward_packed")
    CALLS["fwd packed stored"] += 1
    return o, sT, ws


@gated_delta_fwd_packed_stored.register_fake
def _(q, k, v, g, beta, s0, cu, flags):
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    nbytes = packed_workspace_bytes(N, T, H, HK, DK, DV, True)
    return (q.new_empty(1, T, H, DV), q.new_empty(N, H, DK, DV, dtype=torch.float32),
            q.new_empty(nbytes, dtype=torch.uint8))


def _packed_grads(q, k, v, cu):
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    dev = q.device
    f32 = dict(dtype=torch.float32, device=dev)
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty(1, T, H, **f32),
            torch.empty(1, T, H, **f32), torch.empty(N, H, DK, DV, **f32))


@torch.library.custom_op("macai_b200::gated_delta_bwd_packed", mutates_args=(), device_types="cuda")
def gated_delta_bwd_packed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor, beta: torch.Tensor,
                           s0: Optional[torch.Tensor], cu: torch.Tensor, do: torch.Tensor, dsT: Optional[torch.Tensor],
                           flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                torch.Tensor]:
    """(dq, dk, dv, dg, dbeta, ds0) over packed rows, the chunk states recomputed from the inputs."""
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    lib = _lib.load()
    dev = q.device
    dq, dk, dv, dg, dbeta, ds0 = _packed_grads(q, k, v, cu)
    nbytes = packed_workspace_bytes(N, T, H, HK, DK, DV, True)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.gd_backward_packed(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(s0), _p(do), _p(dsT), _p(dq), _p(dk),
                                    _p(dv), _p(dg), _p(dbeta), _p(ds0), _p(cu), N, _DTYPES[q.dtype], T, H, HK, DK, DV,
                                    flags, _p(ws), nbytes, _stream(dev))
    _lib.check(st, "gd_backward_packed")
    CALLS["bwd packed"] += 1
    return dq, dk, dv, dg, dbeta, ds0


@gated_delta_bwd_packed.register_fake
def _(q, k, v, g, beta, s0, cu, do, dsT, flags):
    return _packed_grads(q, k, v, cu)


# ws is declared unmutated for the reason given at gated_delta_bwd_stored
@torch.library.custom_op("macai_b200::gated_delta_bwd_packed_stored", mutates_args=(), device_types="cuda")
def gated_delta_bwd_packed_stored(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                                  cu: torch.Tensor, do: torch.Tensor, dsT: Optional[torch.Tensor], ws: torch.Tensor,
                                  flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                       torch.Tensor, torch.Tensor]:
    """(dq, dk, dv, dg, dbeta, ds0) over packed rows from the states gated_delta_fwd_packed_stored kept in ws."""
    N, T, H, HK, DK, DV = _pdims(q, v, cu)
    lib = _lib.load()
    dev = q.device
    dq, dk, dv, dg, dbeta, ds0 = _packed_grads(q, k, v, cu)
    with torch.cuda.device(dev):
        st = lib.gd_backward_packed(_p(q), _p(k), _p(v), None, _p(beta), None, _p(do), _p(dsT), _p(dq), _p(dk),
                                    _p(dv), _p(dg), _p(dbeta), _p(ds0), _p(cu), N, _DTYPES[q.dtype], T, H, HK, DK, DV,
                                    flags | _lib.GD_STATES_STORED, _p(ws), ws.numel(), _stream(dev))
    _lib.check(st, "gd_backward_packed")
    CALLS["bwd packed stored"] += 1
    return dq, dk, dv, dg, dbeta, ds0


@gated_delta_bwd_packed_stored.register_fake
def _(q, k, v, beta, cu, do, dsT, ws, flags):
    return _packed_grads(q, k, v, cu)


def _setup_context_packed(ctx, inputs, output):
    q, k, v, g, beta, s0, cu, flags = inputs
    ctx.save_for_backward(q, k, v, g, beta, s0, cu)
    ctx.flags = flags
    ctx.has_s0 = s0 is not None


def _backward_packed(ctx, do, dsT):
    q, k, v, g, beta, s0, cu = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*v.shape, dtype=q.dtype, device=q.device)
    do = do.to(q.dtype).contiguous()
    dsT = None if dsT is None else dsT.to(torch.float32).contiguous()
    dq, dk, dv, dg, dbeta, ds0 = gated_delta_bwd_packed(q, k, v, g, beta, s0, cu, do, dsT, ctx.flags)
    return dq, dk, dv, dg, dbeta, (ds0 if ctx.has_s0 else None), None, None


gated_delta_fwd_packed.register_autograd(_backward_packed, setup_context=_setup_context_packed)


def _setup_context_packed_stored(ctx, inputs, output):
    q, k, v, g, beta, s0, cu, flags = inputs
    ctx.save_for_backward(q, k, v, beta, cu, output[2])
    ctx.flags = flags
    ctx.has_s0 = s0 is not None


def _backward_packed_stored(ctx, do, dsT, _dws):
    q, k, v, beta, cu, ws = ctx.saved_tensors
    if do is None:
        do = torch.zeros(*v.shape, dtype=q.dtype, device=q.device)
    do = do.to(q.dtype).contiguous()
    dsT = None if dsT is None else dsT.to(torch.float32).contiguous()
    dq, dk, dv, dg, dbeta, ds0 = gated_delta_bwd_packed_stored(q, k, v, beta, cu, do, dsT, ws, ctx.flags)
    return dq, dk, dv, dg, dbeta, (ds0 if ctx.has_s0 else None), None, None


gated_delta_fwd_packed_stored.register_autograd(_backward_packed_stored, setup_context=_setup_context_packed_stored)


def check_cu_seqlens(cu_seqlens, T: int, device) -> torch.Tensor:
    """cu_seqlens as the kernels take it (int32 on q's device), after the checks a wrong boundary list needs: 1-D with
    N + 1 >= 2 entries, starting at 0, non-decreasing, ending at T (one host synchronisation for a device tensor)."""
    cu = torch.as_tensor(cu_seqlens)
    if cu.dim() != 1 or cu.numel() < 2:
        raise ValueError(f"cu_seqlens must be 1-D with N + 1 >= 2 entries; got shape {tuple(cu.shape)}")
    if cu.dtype.is_floating_point or cu.dtype == torch.bool:
        raise TypeError(f"cu_seqlens must be an integer tensor; got {cu.dtype}")
    c = cu.to(device=device, dtype=torch.int64)
    ok = torch.stack([c[0] == 0, c[-1] == T, (c[1:] >= c[:-1]).all()]).all()
    if not bool(ok):
        raise ValueError(f"cu_seqlens must start at 0, not decrease and end at the token count T={T}")
    return c.to(torch.int32).contiguous()


def _training(*xs) -> bool:
    """Autograd will record this call (some input needs a gradient)."""
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in xs)


def _forward(q, k, v, g, beta, s0, flags):
    """The forward op for this call: the stored-states one when RECOMPUTE_STATES is False and autograd will record
    the call (the reference keeps states only for a backward, op.py:108, :141-142), else the plain one. A training
    forward keeps the two-CTA state pass (GD_WIDE_STATE_PASS), the one the stored-states forward and the backward's
    recompute run, so that o has the same bits in both modes and however many heads share the call; a forward for
    inference may take the four-CTA pass when its (head, row) pairs leave SMs idle."""
    if _training(q, k, v, g, beta, s0):
        if not RECOMPUTE_STATES:
            o, sT, _ = gated_delta_fwd_stored(q, k, v, g, beta, s0, flags)
            return o, sT
        return gated_delta_fwd(q, k, v, g, beta, s0, flags | _lib.GD_WIDE_STATE_PASS)
    return gated_delta_fwd(q, k, v, g, beta, s0, flags)


def _forward_packed(q, k, v, g, beta, s0, cu, flags):
    """_forward over packed rows."""
    if _training(q, k, v, g, beta, s0):
        if not RECOMPUTE_STATES:
            o, sT, _ = gated_delta_fwd_packed_stored(q, k, v, g, beta, s0, cu, flags)
            return o, sT
        return gated_delta_fwd_packed(q, k, v, g, beta, s0, cu, flags | _lib.GD_WIDE_STATE_PASS)
    return gated_delta_fwd_packed(q, k, v, g, beta, s0, cu, flags)


def _pad_heads(q, k, v, s0, flags):
    """Heads narrower than the built width (multiples of 32 below 128) zero-padded to it, differentiably (autograd
    slices the gradients back): zero key dimensions change neither the l2 norms nor the states, zero value columns stay
    zero, and the query scale keeps the caller's key width (GD_KEY_WIDTH). Returns the padded tensors, the flags and
    the caller's (DK, DV), or the inputs unchanged when they are built-width already."""
    DK, DV, W = q.shape[-1], v.shape[-1], max(HEAD_DIMS)
    if DK == W and DV == W:
        return q, k, v, s0, flags, None
    pad = torch.nn.functional.pad
    q, k, v = pad(q, (0, W - DK)), pad(k, (0, W - DK)), pad(v, (0, W - DV))
    s0 = None if s0 is None else pad(s0, (0, W - DV, 0, W - DK))
    if flags & _lib.GD_SCALE_Q:
        flags |= _lib.GD_KEY_WIDTH(DK)
    return q, k, v, s0, flags, (DK, DV)


def _unpad(o, sT, widths):
    """The outputs of a padded call cut back to the caller's widths."""
    if widths is None:
        return o, sT
    DK, DV = widths
    return o[..., :DV], (None if sT is None else sT[..., :DK, :DV])


# ------------------------------------------------------------------------------------------------------------------
# the reference's Python surface

class GatedDeltaRule:
    """o, S_T = recurrence(q, k, v, g, beta, S_0) on [B, T, H, D] tensors with q already normalised and scaled, as the
    reference's autograd function (op.py:116-257): `GatedDeltaRule.apply(q, k, v, g, beta, s0, save)`. `save` is
    accepted for signature compatibility; autograd records the op whenever an input requires grad. The backward
    recomputes the chunk states unless RECOMPUTE_STATES is False (the reference's setting, op.py:27-33)."""

    @staticmethod
    def apply(q, k, v, g, beta, s0, save: bool = True):
        dt = q.dtype
        check_dtype(dt)
        k, v = k.to(dt), v.to(dt)
        check_shapes(q, k, v, g, beta, s0)
        q, k, v, s0, flags, widths = _pad_heads(q, k, v, None if s0 is None else s0.float(), 0)
        o, sT = _forward(q.contiguous(), k.contiguous(), v.contiguous(), g.float().contiguous(),
                         beta.float().contiguous(), None if s0 is None else s0.contiguous(), flags)
        return _unpad(o, sT, widths)


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + eps) over the last dimension (the reference's op.py:260-261; transformers' l2norm)."""
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def chunk_gated_delta_rule(query, key, value, g, beta, chunk_size: int = 64, initial_state=None,
                           output_final_state: bool = False, use_qk_l2norm_in_kernel: bool = False, **kwargs):
    """Drop-in for transformers' torch_chunk_gated_delta_rule: query, key [B, T, HK, DK]; value [B, T, H, DV]
    (H = HK, or a multiple of it: each key head then serves H / HK consecutive value heads); g (log decay, <= 0) and
    beta [B, T, H]; initial_state [B, H, DK, DV] or None. Returns the output [B, T, H, DV] in the query's dtype and the
    final state (float32) when output_final_state, else None. chunk_size is accepted and not used (the kernels chunk by
    64 tokens), as in the reference (op.py:264-269). cu_seqlens (packed rows: batch size 1, N sequences along the
    tokens, initial_state and the final state [N, H, DK, DV]) runs every sequence as its own row, with fla's
    semantics; the reference refuses it (op.py:270-273)."""
    cu_seqlens = kwargs.get("cu_seqlens")
    dt = query.dtype
    check_dtype(dt)
    # the kernels read q, k, v in one dtype: key and value follow the query's (differentiably, so their gradients
    # come back in their own dtypes)
    k, v = key.to(dt), value.to(dt)
    flags = _lib.GD_SCALE_Q | (_lib.GD_L2NORM if use_qk_l2norm_in_kernel else 0)
    if cu_seqlens is not None:
        # packed rows: one batch row holding N sequences, each with its own state (initial_state [N, H, DK, DV])
        if query.dim() != 4 or query.shape[0] != 1:
            raise ValueError(f"with cu_seqlens the batch size must be 1 (sequences packed along the tokens); got "
                             f"query {tuple(query.shape)}")
        cu = check_cu_seqlens(cu_seqlens, query.shape[1], query.device)
        N = cu.numel() - 1
        B, T, H, HK, DK, DV = _dims(query, v)
        if initial_state is not None and initial_state.shape != (N, H, DK, DV):
            raise ValueError(f"with cu_seqlens initial_state must be [N, H, DK, DV] = {(N, H, DK, DV)}; got "
                             f"{tuple(initial_state.shape)}")
        check_shapes(query, k, v, g, beta, None)
        s0 = None if initial_state is None else initial_state.to(torch.float32)
        q, k, v, s0, flags, widths = _pad_heads(query, k, v, s0, flags)
        o, sT = _forward_packed(q.contiguous(), k.contiguous(), v.contiguous(), g.to(torch.float32).contiguous(),
                                beta.to(torch.float32).contiguous(), None if s0 is None else s0.contiguous(), cu,
                                flags)
        o, sT = _unpad(o, sT, widths)
        return o, (sT if output_final_state else None)
    check_shapes(query, k, v, g, beta, initial_state)
    s0 = None if initial_state is None else initial_state.to(torch.float32)
    q, k, v, s0, flags, widths = _pad_heads(query, k, v, s0, flags)
    o, sT = _forward(q.contiguous(), k.contiguous(), v.contiguous(), g.to(torch.float32).contiguous(),
                     beta.to(torch.float32).contiguous(), None if s0 is None else s0.contiguous(), flags)
    o, sT = _unpad(o, sT, widths)
    return o, (sT if output_final_state else None)


def recurrent_reference(q, k, v, g, beta, s0):
    """The recurrence step by step in plain PyTorch ([B, T, H, D] inputs, q already normalised and scaled), the
    reference's parity utility (op.py:301-314) kept for users' own checks. Not used by the ops."""
    s = s0.clone()
    outs = []
    for t in range(q.shape[1]):
        a = g[:, t].exp()[..., None, None]
        st = s * a
        u = (st * k[:, t, :, :, None]).sum(-2)
        d = beta[:, t, :, None] * (v[:, t] - u)
        s = st + k[:, t, :, :, None] * d[:, :, None, :]
        outs.append((s * q[:, t, :, :, None]).sum(-2))
    return torch.stack(outs, 1), s
