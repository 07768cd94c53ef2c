"""The convolution-path oracle (oracle/conv_f64.py) pinned on CPU against the reference's own float64 truth for this
part, restated (tests/test_layer.py:232-252 of the reference: F.conv1d with padding 3 over the channel-first
transpose, SiLU, split, reshape, repeat_interleave), and its backward against float64 autograd of that expression."""
import pytest
import torch
import torch.nn.functional as F

from oracle import conv_f64

# (key_dim, key head width, rep, value head width): a small GQA case and a plain one
CASES = [(16, 8, 2, 8), (24, 8, 1, 12)]


def truth(x, w, kd, dk, rep, dv):
    B, T, C = x.shape
    u = F.conv1d(x.transpose(1, 2), w, padding=3, groups=C)[:, :, :T]
    y = F.silu(u).transpose(1, 2)
    q, k, v = torch.split(y, [kd, kd, C - 2 * kd], dim=-1)
    q = q.reshape(B, T, -1, dk).repeat_interleave(rep, dim=2)
    k = k.reshape(B, T, -1, dk).repeat_interleave(rep, dim=2)
    return q, k, v.reshape(B, T, -1, dv)


def make(kd, dk, rep, dv, B=2, T=37, seed=0):
    hv = kd // dk * rep
    C = 2 * kd + hv * dv
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, C, generator=gen, dtype=torch.float64)
    w = torch.randn(C, 1, 4, generator=gen, dtype=torch.float64) * 0.3
    return x, w


@pytest.mark.parametrize("case", CASES, ids=str)
def test_forward_matches_conv1d(case):
    x, w = make(*case)
    for a, b in zip(conv_f64.forward(x, w, *case), truth(x, w, *case)):
        assert a.shape == b.shape and torch.allclose(a, b, rtol=1e-13, atol=1e-14)


@pytest.mark.parametrize("case", CASES, ids=str)
def test_backward_matches_float64_autograd(case):
    x, w = make(*case, seed=1)
    xs, ws = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    outs = truth(xs, ws, *case)
    gen = torch.Generator().manual_seed(2)
    gouts = [torch.randn(o.shape, generator=gen, dtype=torch.float64) for o in outs]
    gx, gw = torch.autograd.grad(sum((o * g).sum() for o, g in zip(outs, gouts)), (xs, ws))
    dx, dw = conv_f64.backward(x, w, *gouts, *case)
    assert torch.allclose(dx, gx, rtol=1e-12, atol=1e-12)
    assert torch.allclose(dw, gw.reshape(-1, 4), rtol=1e-12, atol=1e-12)


def test_missing_cotangents_are_zero():
    case = CASES[0]
    x, w = make(*case, seed=3)
    q, k, v = conv_f64.forward(x, w, *case)
    gen = torch.Generator().manual_seed(4)
    gv = torch.randn(v.shape, generator=gen, dtype=torch.float64)
    a = conv_f64.backward(x, w, None, None, gv, *case)
    b = conv_f64.backward(x, w, torch.zeros_like(q), torch.zeros_like(k), gv, *case)
    assert all(torch.equal(u, v) for u, v in zip(a, b))
