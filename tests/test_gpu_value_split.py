"""The forward state pass's value split (the reference's VALUE_SPLIT rule, src/macai/gated_delta/op.py:75-87: the
split grows when the (batch, head) grid alone leaves SMs idle). gd_fwd_state runs four CTAs per (head, row) with 32
value columns each when 4 x heads x rows fit on the GPU at once, else two CTAs of 64 columns; GD_WIDE_STATE_PASS forces
two. The two forms form the same products and apply the same epilogue arithmetic, but with tokens on the tensor core's
M side instead of value columns its fp32 sums round differently in the last bits: both are held to the parity bar and
to each other within a rounding-level tolerance (a given split is bitwise deterministic, tests/test_gpu_backward.py)."""
import ctypes

import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref
from test_gpu_forward import inputs

pytestmark = pytest.mark.gpu


def forward_abi(q, k, v, g, beta, s0, wide):
    """gd_prep + gd_fwd_state through the C ABI (the drop-in's normalisation and query scale), with or without
    GD_WIDE_STATE_PASS; returns o and the final state."""
    from macai_b200 import _lib
    lib = _lib.load()
    dev = "cuda"
    B, T, H, D = v.shape
    HK = q.shape[2]
    q, k, v = (x.to(dev).contiguous() for x in (q, k, v))
    g, beta = g.to(dev).float().contiguous(), beta.to(dev).float().contiguous()
    s0d = None if s0 is None else s0.to(dev).float().contiguous()
    flags = _lib.GD_L2NORM | _lib.GD_SCALE_Q
    nb = lib.gd_workspace_bytes(B, T, H, HK, D, D, 0)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    o = torch.empty(B, T, H, D, dtype=q.dtype, device=dev)
    sT = torch.empty(B, H, D, D, dtype=torch.float32, device=dev)
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dt = _lib.GD_BFLOAT16
    _lib.check(lib.gd_prep(P(q), P(k), P(v), P(g), P(beta), dt, B, T, H, HK, D, D, flags, P(ws), nb, st), "prep")
    f = flags | (_lib.GD_WIDE_STATE_PASS if wide else 0)
    _lib.check(lib.gd_fwd_state(P(s0d), P(o), P(sT), dt, B, T, H, HK, D, D, f, P(ws), nb, st), "fwd_state")
    torch.cuda.synchronize()
    assert lib.gd_read_error(P(ws), st, None) == 0
    return o.cpu(), sT.cpu()


@pytest.mark.parametrize("shape", [(1, 300, 4, 4), (2, 130, 4, 2), (1, 1, 1, 1), (1, 2048, 2, 2)])
def test_narrow_matches_wide(shape):
    """Four CTAs per (head, row) (the automatic choice at these sizes) against two: both meet the bar against float64,
    and they differ by rounding only (relative to the output's scale)."""
    B, T, H, HK = shape
    q, k, v, g, beta, s0 = inputs(B, T, H, seed=3 * T + H, HK=HK)
    narrow = forward_abi(q, k, v, g, beta, s0, wide=False)
    wide = forward_abi(q, k, v, g, beta, s0, wide=True)
    truth = ref.dropin(q, k, v, g, beta, s0)
    theirs = transformers_ref.run(q, k, v, g, beta, s0)
    for got in (narrow, wide):
        rep = parity.check(list(got), list(theirs[:2]), list(truth[:2]), names=("o", "sT"))
        assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}
    for a, b in zip(narrow, wide):
        scale = b.float().abs().max().item()
        assert (a.float() - b.float()).abs().max().item() <= 2e-2 * scale


def test_narrow_parity():
    """The narrow pass against float64 with the north star's bar (o and the final state)."""
    q, k, v, g, beta, s0 = inputs(1, 700, 3, seed=41)
    got = forward_abi(q, k, v, g, beta, s0, wide=False)
    truth = ref.dropin(q, k, v, g, beta, s0)
    theirs = transformers_ref.run(q, k, v, g, beta, s0)
    rep = parity.check(list(got), list(theirs[:2]), list(truth[:2]), names=("o", "sT"))
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}
