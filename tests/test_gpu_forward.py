"""The forward (o, S_T) of the B200 kernels through the drop-in against the float64 oracle, with the parity bar of
the north star: max error <= 2x transformers' own error against float64 on the same inputs (oracle/parity.py)."""
import math

import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref

pytestmark = pytest.mark.gpu


def inputs(B, T, H, D=128, seed=0, s0=True, HK=None, dtype=torch.bfloat16):
    """BASELINE.json's configs[0] distributions: q, k, v ~ N(0,1); beta = sigmoid(N(0,1));
    g = -exp(U(log 1, log 16)) * softplus(N(0,1))."""
    HK = HK or H
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, HK, D, generator=gen).to(dtype)
    k = torch.randn(B, T, HK, D, generator=gen).to(dtype)
    v = torch.randn(B, T, H, D, generator=gen).to(dtype)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    g = -torch.exp(torch.rand(B, T, H, generator=gen) * math.log(16.0)) * torch.nn.functional.softplus(
        torch.randn(B, T, H, generator=gen))
    st = torch.randn(B, H, D, D, generator=gen) * 0.02 if s0 else None
    return q, k, v, g, beta, st


def run_dropin(q, k, v, g, beta, s0):
    from macai_b200.gated_delta import chunk_gated_delta_rule
    dev = "cuda"
    o, sT = chunk_gated_delta_rule(q.to(dev), k.to(dev), v.to(dev), g.to(dev), beta.to(dev),
                                   initial_state=None if s0 is None else s0.to(dev), output_final_state=True,
                                   use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    return o.cpu(), sT.cpu()


@pytest.mark.parametrize("shape", [(1, 64, 1), (1, 1, 1), (1, 100, 2), (2, 256, 3), (1, 1000, 2), (2, 65, 2)])
def test_forward_parity(shape):
    B, T, H = shape
    q, k, v, g, beta, s0 = inputs(B, T, H, seed=T + H)
    o, sT = run_dropin(q, k, v, g, beta, s0)
    assert o.dtype == torch.bfloat16 and sT.dtype == torch.float32
    truth = ref.dropin(q, k, v, g, beta, s0)
    theirs = transformers_ref.run(q, k, v, g, beta, s0)
    rep = parity.check([o, sT], theirs, truth, names=("o", "sT"))
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


def test_forward_no_initial_state():
    q, k, v, g, beta, _ = inputs(1, 200, 2, seed=5, s0=False)
    o, sT = run_dropin(q, k, v, g, beta, None)
    truth = ref.dropin(q, k, v, g, beta, None)
    theirs = transformers_ref.run(q, k, v, g, beta, None)
    rep = parity.check([o, sT], theirs, truth, names=("o", "sT"))
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}
