"""The stored-states mode (RECOMPUTE_STATES = False: the training forward keeps the chunk matrices, states and Vn for
the backward, which then skips the recompute) against the default recompute mode: every output and every gradient
must be the same bits, as the reference's tests/test_memory.py:100-109 requires of its recompute and stored designs."""
import pytest
import torch

from oracle import parity
from test_gpu_backward import run_grads
from test_gpu_forward import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture
def op_module():
    from macai_b200.gated_delta import op
    saved = op.RECOMPUTE_STATES
    yield op
    op.RECOMPUTE_STATES = saved


def case(B, T, H, seed, s0=True, HK=None):
    q, k, v, g, beta, st = inputs(B, T, H, seed=seed, s0=s0, HK=HK)
    gen = torch.Generator().manual_seed(seed + 500)
    do = torch.randn(B, T, H, 128, generator=gen).to(torch.bfloat16)
    dsT = torch.randn(B, H, 128, 128, generator=gen) * 0.1
    return q, k, v, g, beta, st, do, dsT


@pytest.mark.parametrize("shape", [(2, 300, 4, 2, True), (1, 128, 2, 2, False), (1, 65, 3, 3, True)])
def test_stored_states_give_the_recompute_bits(op_module, shape):
    B, T, H, HK, s0 = shape
    x = case(B, T, H, seed=T + H, s0=s0, HK=HK)
    op_module.RECOMPUTE_STATES = True
    before = dict(op_module.CALLS)
    recomputed = run_grads(*x)
    op_module.RECOMPUTE_STATES = False
    stored = run_grads(*x)
    assert op_module.CALLS["fwd stored"] == before.get("fwd stored", 0) + 1
    assert op_module.CALLS["bwd stored"] == before.get("bwd stored", 0) + 1
    for name, a, b in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), recomputed, stored):
        assert (a is None and b is None) or parity.identical(a, b), name


def test_stored_states_survive_a_second_backward(op_module):
    """retain_graph: the second backward reads the same kept states and gives the same gradients."""
    from macai_b200.gated_delta import chunk_gated_delta_rule
    op_module.RECOMPUTE_STATES = False
    q, k, v, g, beta, st, do, dsT = case(1, 200, 2, seed=3)
    xs = [t.cuda().requires_grad_(True) for t in (q, k, v, g, beta)]
    o, sT = chunk_gated_delta_rule(*xs, initial_state=st.cuda(), output_final_state=True,
                                   use_qk_l2norm_in_kernel=True)
    loss = (o.float() * do.cuda().float()).sum() + (sT * dsT.cuda()).sum()
    first = torch.autograd.grad(loss, xs, retain_graph=True)
    second = torch.autograd.grad(loss, xs)
    for a, b in zip(first, second):
        assert parity.identical(a.cpu(), b.cpu())


def test_inference_forward_keeps_nothing(op_module):
    """Without autograd recording the call the plain forward runs (no workspace kept), as the reference's
    keeps_nothing (op.py:108)."""
    from macai_b200.gated_delta import chunk_gated_delta_rule
    op_module.RECOMPUTE_STATES = False
    q, k, v, g, beta, st, _, _ = case(1, 100, 2, seed=4)
    before = dict(op_module.CALLS)
    with torch.no_grad():
        chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=st.cuda(),
                               use_qk_l2norm_in_kernel=True)
    assert op_module.CALLS["fwd"] == before.get("fwd", 0) + 1
    assert op_module.CALLS.get("fwd stored", 0) == before.get("fwd stored", 0)
