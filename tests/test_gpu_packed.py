"""Packed rows (cu_seqlens) through the drop-in: N sequences along the tokens of one batch row, each run as its own
row (fla's semantics; the reference refuses cu_seqlens, src/macai/gated_delta/op.py:270-273).

- The packed call gives the same bits as N separate calls (forward o and S_T, every gradient): each sequence starts
  a new chunk, so every chunk computes exactly what the separate call computes.
- Against float64 (oracle.gated_delta_f64.dropin_packed, pinned on CPU to a token recurrence with state resets) with
  the north star's bar: error <= 2x that of transformers' function run sequence by sequence.
- The stored-states mode gives the same bits as the recompute mode; sequences without tokens pass their state (and
  its gradient) through."""
import math

import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref

pytestmark = pytest.mark.gpu


def inputs(T, H, HK, N, D=128, seed=0, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, T, HK, D, generator=gen).to(dtype)
    k = torch.randn(1, T, HK, D, generator=gen).to(dtype)
    v = torch.randn(1, T, H, D, generator=gen).to(dtype)
    beta = torch.sigmoid(torch.randn(1, T, H, generator=gen))
    g = -torch.exp(torch.rand(1, T, H, generator=gen) * math.log(16.0)) * torch.nn.functional.softplus(
        torch.randn(1, T, H, generator=gen))
    s0 = torch.randn(N, H, D, D, generator=gen) * 0.02
    do = torch.randn(1, T, H, D, generator=gen).to(dtype)
    dsT = torch.randn(N, H, D, D, generator=gen) * 0.1
    return q, k, v, g, beta, s0, do, dsT


def cu_of(lengths):
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + n)
    return cu


def run(q, k, v, g, beta, s0, do, dsT, cu=None):
    """Forward and backward through the drop-in on the GPU: (o, S_T, dq, dk, dv, dg, dbeta, ds0) on the CPU."""
    from macai_b200.gated_delta import chunk_gated_delta_rule
    xs = [t.cuda().requires_grad_(True) for t in (q, k, v, g, beta, s0)]
    kw = {} if cu is None else {"cu_seqlens": torch.tensor(cu, dtype=torch.int32, device="cuda")}
    o, sT = chunk_gated_delta_rule(*xs[:5], initial_state=xs[5], output_final_state=True,
                                   use_qk_l2norm_in_kernel=True, **kw)
    torch.autograd.backward([o, sT], [do.cuda(), dsT.cuda()])
    torch.cuda.synchronize()
    return [o.detach().cpu(), sT.detach().cpu()] + [x.grad.cpu() for x in xs]


def separate(q, k, v, g, beta, s0, do, dsT, lengths):
    """The same sequences as N separate calls (a sequence without tokens: its state and gradient pass through)."""
    outs = []
    cu = cu_of(lengths)
    for n, L in enumerate(lengths):
        a, b = cu[n], cu[n + 1]
        if L == 0:
            e = lambda x: x[:, a:a]
            outs.append([e(v), s0[n:n + 1], e(q), e(k), e(v), e(g), e(beta), dsT[n:n + 1]])
            continue
        sl = slice(a, b)
        outs.append(run(q[:, sl], k[:, sl], v[:, sl], g[:, sl], beta[:, sl], s0[n:n + 1], do[:, sl], dsT[n:n + 1]))
    cat = lambda i: torch.cat([o[i] for o in outs], dim=1)
    stack = lambda i: torch.cat([o[i] for o in outs], dim=0)
    return [cat(0), stack(1), cat(2), cat(3), cat(4), cat(5), cat(6), stack(7)]


NAMES = ("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0")


@pytest.mark.parametrize("lengths,H,HK", [
    ([1, 63, 64, 65, 0, 200, 130], 4, 2),     # one-token, chunk-exact, ragged, empty; GQA
    ([300], 2, 2),                           # one sequence = the plain call
    ([17] * 40, 2, 1),                       # many short sequences, GQA 2:1
], ids=["ragged_gqa", "single", "many_short"])
def test_packed_equals_separate_calls_bitwise(lengths, H, HK):
    T = sum(lengths)
    q, k, v, g, beta, s0, do, dsT = inputs(T, H, HK, len(lengths), seed=len(lengths) + H)
    got = run(q, k, v, g, beta, s0, do, dsT, cu_of(lengths))
    want = separate(q, k, v, g, beta, s0, do, dsT, lengths)
    for name, a, b in zip(NAMES, got, want):
        assert a.shape == b.shape, name
        assert parity.identical(a, b), (name, (a.double() - b.double()).abs().max().item())


def test_packed_parity_against_float64():
    lengths = [100, 37, 0, 300, 64]
    T, H = sum(lengths), 2
    q, k, v, g, beta, s0, do, dsT = inputs(T, H, H, len(lengths), seed=3)
    cu = cu_of(lengths)
    got = run(q, k, v, g, beta, s0, do, dsT, cu)
    truth = ref.dropin_packed(q, k, v, g, beta, cu, s0, do.double(), dsT.double())
    parts = []
    for n, L in enumerate(lengths):  # transformers' function, sequence by sequence
        a, b = cu[n], cu[n + 1]
        if L == 0:
            e = lambda x: x[:, a:a]
            parts.append([e(v), s0[n:n + 1], e(q), e(k), e(v), e(g), e(beta), dsT[n:n + 1]])
            continue
        sl = slice(a, b)
        parts.append(list(transformers_ref.run(q[:, sl], k[:, sl], v[:, sl], g[:, sl], beta[:, sl], s0[n:n + 1],
                                               do[:, sl], dsT[n:n + 1])))
    theirs = [torch.cat([p[i] for p in parts], dim=1 if i not in (1, 7) else 0) for i in range(8)]
    rep = parity.check(got, theirs, truth, names=NAMES)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


def test_packed_stored_mode_same_bits():
    from macai_b200.gated_delta import op
    lengths = [70, 5, 128, 1]
    T, H = sum(lengths), 2
    q, k, v, g, beta, s0, do, dsT = inputs(T, H, H, len(lengths), seed=9)
    cu = cu_of(lengths)
    a = run(q, k, v, g, beta, s0, do, dsT, cu)
    op.RECOMPUTE_STATES = False
    try:
        calls = op.CALLS["fwd packed stored"]
        b = run(q, k, v, g, beta, s0, do, dsT, cu)
        assert op.CALLS["fwd packed stored"] == calls + 1
    finally:
        op.RECOMPUTE_STATES = True
    for name, x, y in zip(NAMES, a, b):
        assert parity.identical(x, y), name


def test_packed_forward_only_and_int64_boundaries():
    """No gradients (the forward-only workspace), boundaries given as an int64 tensor (as transformers passes them)."""
    from macai_b200.gated_delta import chunk_gated_delta_rule
    lengths = [10, 90, 3]
    T, H = sum(lengths), 2
    q, k, v, g, beta, s0, _, _ = inputs(T, H, H, len(lengths), seed=11)
    cu = torch.tensor(cu_of(lengths), dtype=torch.int64, device="cuda")
    with torch.no_grad():
        o, sT = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=s0.cuda(),
                                       output_final_state=True, use_qk_l2norm_in_kernel=True, cu_seqlens=cu)
    # the separate calls forward-only as well (a forward for inference may take the four-CTA state pass, a training
    # forward keeps the two-CTA one)
    outs = []
    with torch.no_grad():
        for n, (a, b) in enumerate(zip(cu_of(lengths)[:-1], cu_of(lengths)[1:])):
            sl = slice(a, b)
            outs.append(chunk_gated_delta_rule(q[:, sl].cuda(), k[:, sl].cuda(), v[:, sl].cuda(), g[:, sl].cuda(),
                                               beta[:, sl].cuda(), initial_state=s0[n:n + 1].cuda(),
                                               output_final_state=True, use_qk_l2norm_in_kernel=True))
    want = (torch.cat([x[0].cpu() for x in outs], dim=1), torch.cat([x[1].cpu() for x in outs], dim=0))
    assert parity.identical(o.cpu(), want[0]) and parity.identical(sT.cpu(), want[1])
