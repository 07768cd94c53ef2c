"""Head widths below the built 128 (multiples of 32, as the reference takes, src/macai/gated_delta/op.py:124-125): the
drop-in zero-pads q, k, v and the state to 128 (zero key dimensions change neither the l2 norms nor the states, zero
value columns stay zero) and keeps the query scale at the caller's key width; forward and backward against the float64
oracle with the north star's bar, at the caller's widths."""
import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref
from test_gpu_backward import NAMES, run_grads
from test_gpu_forward import inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dk,dv", [(64, 64), (32, 128), (128, 96), (96, 32)])
def test_padded_widths_parity(dk, dv):
    B, T, H = 2, 150, 2
    q, k, v, g, beta, s0 = inputs(B, T, H, seed=dk + dv)
    q, k, v = q[..., :dk].contiguous(), k[..., :dk].contiguous(), v[..., :dv].contiguous()
    s0 = s0[:, :, :dk, :dv].contiguous()
    gen = torch.Generator().manual_seed(dk * dv)
    do = torch.randn(B, T, H, dv, generator=gen).to(torch.bfloat16)
    dsT = torch.randn(B, H, dk, dv, generator=gen) * 0.1
    got = run_grads(q, k, v, g, beta, s0, do, dsT)
    assert got[0].shape == (B, T, H, dv) and got[1].shape == (B, H, dk, dv) and got[2].shape == q.shape
    truth = ref.dropin(q, k, v, g, beta, s0, do.double(), dsT)
    theirs = transformers_ref.run(q, k, v, g, beta, s0, do=do, dsT=dsT)
    rep = parity.check(got, theirs, truth, names=NAMES)
    assert not parity.failures(rep), {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}
