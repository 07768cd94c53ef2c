"""Forward + backward of the B200 kernels through the drop-in (autograd), every gradient against the float64 oracle,
with the north star's bar: max error <= 2x transformers' own error against float64 on the same inputs."""
import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref
from test_gpu_forward import inputs

pytestmark = pytest.mark.gpu
NAMES = ("o", "sT", "dquery", "dkey", "dvalue", "dg", "dbeta", "ds0")


def run_grads(q, k, v, g, beta, s0, do, dsT):
    from macai_b200.gated_delta import chunk_gated_delta_rule
    dev = "cuda"
    xs = [t.to(dev).requires_grad_(True) for t in (q, k, v, g, beta)]
    s0d = None if s0 is None else s0.to(dev).requires_grad_(True)
    o, sT = chunk_gated_delta_rule(*xs, initial_state=s0d, output_final_state=True, use_qk_l2norm_in_kernel=True)
    loss = (o.float() * do.to(dev).float()).sum()
    if dsT is not None:
        loss = loss + (sT * dsT.to(dev)).sum()
    loss.backward()
    torch.cuda.synchronize()
    grads = [x.grad.cpu() for x in xs] + [None if s0d is None else s0d.grad.cpu()]
    return [o.detach().cpu(), sT.detach().cpu()] + grads


def check_case(B, T, H, seed, s0=True, HK=None):
    q, k, v, g, beta, st = inputs(B, T, H, seed=seed, s0=s0, HK=HK)
    gen = torch.Generator().manual_seed(seed + 1000)
    do = torch.randn(B, T, H, 128, generator=gen).to(torch.bfloat16)
    dsT = torch.randn(B, H, 128, 128, generator=gen) * 0.1
    got = run_grads(q, k, v, g, beta, st, do, dsT)
    truth = ref.dropin(q, k, v, g, beta, st, do.double(), dsT)
    theirs = transformers_ref.run(q, k, v, g, beta, st, do=do, dsT=dsT)
    rep = parity.check(got, theirs, truth, names=NAMES)
    return rep


@pytest.mark.parametrize("shape", [(1, 64, 1), (1, 1, 1), (1, 100, 2), (2, 130, 2), (1, 512, 2), (2, 65, 3)])
def test_backward_parity(shape):
    B, T, H = shape
    rep = check_case(B, T, H, seed=7 * T + H)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


def test_backward_no_initial_state():
    rep = check_case(1, 200, 2, seed=11, s0=False)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


def test_backward_gqa():
    """16 key heads serving 32 value heads in the 9B model; here 2 key heads serving 4 value heads."""
    rep = check_case(1, 150, 4, seed=13, HK=2)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


def test_backward_is_deterministic():
    """One writer per gradient element, no atomics: repeated runs give the same bits
    (the reference's tests/test_harness.py:196-211)."""
    q, k, v, g, beta, st = inputs(2, 100, 2, seed=5)
    gen = torch.Generator().manual_seed(9)
    do = torch.randn(2, 100, 2, 128, generator=gen).to(torch.bfloat16)
    dsT = torch.randn(2, 2, 128, 128, generator=gen) * 0.1
    runs = [run_grads(q, k, v, g, beta, st, do, dsT) for _ in range(3)]
    for i in (1, 2):
        for a, b in zip(runs[0], runs[i]):
            assert parity.identical(a, b)


def test_backward_many_heads():
    """B * H = 80 value heads (160 state-pass CTAs on 148 SMs: a second wave): forward and backward against float64
    with the bar, and bitwise equal to half of the heads run alone (80 CTAs, one wave; both head counts take the
    two-CTA state pass, so the same arithmetic runs on every head)."""
    q, k, v, g, beta, st = inputs(1, 130, 80, seed=17)
    gen = torch.Generator().manual_seed(18)
    do = torch.randn(1, 130, 80, 128, generator=gen).to(torch.bfloat16)
    dsT = torch.randn(1, 80, 128, 128, generator=gen) * 0.1
    got = run_grads(q, k, v, g, beta, st, do, dsT)
    truth = ref.dropin(q, k, v, g, beta, st, do.double(), dsT)
    theirs = transformers_ref.run(q, k, v, g, beta, st, do=do, dsT=dsT)
    rep = parity.check(got, theirs, truth, names=NAMES)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}
    sl = slice(40, 80)   # half of the heads alone
    few = run_grads(q[:, :, sl], k[:, :, sl], v[:, :, sl], g[:, :, sl], beta[:, :, sl], st[:, sl], do[:, :, sl],
                    dsT[:, sl])
    part = lambda x, dim: x.narrow(dim, 40, 40)
    dims = (2, 1, 2, 2, 2, 2, 2, 1)   # head dimension of o, S_T, dq, dk, dv, dg, dbeta, ds0
    for a, b, d in zip(got, few, dims):
        assert parity.identical(part(a, d), b)
