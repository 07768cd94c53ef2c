"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the third-party "reference torch implementation".

transformers' torch_chunk_gated_delta_rule (transformers/models/qwen3_5/modeling_qwen3_5.py, the function the
reference's drop-in replaces: src/macai/patch.py:27-29; pinned transformers==5.22.1 at requirements.txt:4, 5.5.0 in
this image) is run here on the CPU, forward with autograd plus backward. It is used two ways:
- its error against float64 defines the parity bar (the new kernels must be within 2x of it, per tensor);
- it is the timed CPU baseline (`bench.py --impl reference` and the `cpu_baseline` field).
Only the call sites cited by the reference are used: tests/test_gated_delta.py:37-56, bench/bench_gated_delta.py:160-162.
"""
from __future__ import annotations

import torch


def rule():
    """The installed transformers function (unwrapped if decorated)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mod
    f = mod.torch_chunk_gated_delta_rule
    return getattr(f, "__wrapped__", f)


def _repeat(x, rep):
    return x.repeat_interleave(rep, dim=2) if rep > 1 else x


def run(query, key, value, g, beta, initial_state=None, do=None, dsT=None, output_final_state=True,
        use_qk_l2norm_in_kernel=True, chunk_size=64):
    """Run the transformers function on CPU copies of the inputs, in their own dtypes (q/k/v bf16 stay bf16, so its
    l2norm runs in bf16 as in a real bf16 model). GQA (value heads > key heads) is expanded by repeat_interleave first,
    as the Qwen3.5 layer does (TF modeling_qwen3_5.py:494-496), and the key-side gradients are summed back through it.

    Returns (o, S_T) or, with `do`, (o, S_T, dquery, dkey, dvalue, dg, dbeta, ds0); gradients in the inputs' dtypes."""
    f = rule()
    rep = value.shape[2] // query.shape[2]
    grads = do is not None
    xs = [t.detach().cpu().clone().requires_grad_(grads) for t in (query, key, value, g, beta)]
    s0 = None
    if initial_state is not None:
        s0 = initial_state.detach().cpu().clone().requires_grad_(grads)
    with torch.set_grad_enabled(grads):
        o, sT = f(_repeat(xs[0], rep), _repeat(xs[1], rep), xs[2], xs[3], xs[4], chunk_size=chunk_size,
                  initial_state=s0, output_final_state=True, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
        if not grads:
            return o.detach(), (sT.detach() if output_final_state else None)
        loss = (o.float() * do.detach().cpu().float()).sum()
        if dsT is not None:
            loss = loss + (sT.float() * dsT.detach().cpu().float()).sum()
        loss.backward()
    ds0 = s0.grad if s0 is not None else None
    return (o.detach(), sT.detach(), *(x.grad for x in xs), ds0)
