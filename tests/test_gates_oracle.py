"""The gates oracle (oracle/gates_f64.py) pinned on CPU to the PyTorch expression the reference's gates kernels replace
(transformers' Qwen3.5 layer: beta = b.sigmoid(), g = -A_log.float().exp() * softplus(a.float() + dt_bias); the
reference's docstring, src/macai/layer/_gates.py:1-13) and to float64 autograd of it for the backward."""
import torch
import torch.nn.functional as F

from oracle import gates_f64


def make(shape=(2, 50, 16), seed=0):
    gen = torch.Generator().manual_seed(seed)
    H = shape[-1]
    b = torch.randn(shape, generator=gen, dtype=torch.float64) * 3
    a = torch.randn(shape, generator=gen, dtype=torch.float64) * 8   # reaches past the softplus threshold of 20
    A_log = torch.log(torch.empty(H, dtype=torch.float64).uniform_(1, 16, generator=gen))
    dt_bias = torch.randn(H, generator=gen, dtype=torch.float64) * 4
    return b, a, A_log, dt_bias


def test_forward_matches_the_pytorch_expression():
    b, a, A_log, dt_bias = make()
    beta, g = gates_f64.forward(b, a, A_log, dt_bias)
    assert torch.allclose(beta, b.sigmoid(), rtol=0, atol=1e-15)
    g_ref = -A_log.exp() * F.softplus(a + dt_bias)  # threshold 20 by default
    assert torch.allclose(g, g_ref, rtol=1e-14, atol=1e-14)
    assert ((a + dt_bias) > 20).any() and ((a + dt_bias) < -20).any()


def test_backward_matches_float64_autograd():
    b, a, A_log, dt_bias = make(seed=1)
    xs = [t.clone().requires_grad_(True) for t in (b, a, A_log, dt_bias)]
    beta = xs[0].sigmoid()
    g = -xs[2].exp() * F.softplus(xs[1] + xs[3])
    gen = torch.Generator().manual_seed(2)
    dbeta = torch.randn(beta.shape, generator=gen, dtype=torch.float64)
    dg = torch.randn(g.shape, generator=gen, dtype=torch.float64)
    grads = torch.autograd.grad((beta * dbeta).sum() + (g * dg).sum(), xs)
    mine = gates_f64.backward(b, a, A_log, dt_bias, dbeta, dg)
    for name, x, y in zip(("db", "da", "dA_log", "ddt_bias"), mine, grads):
        assert torch.allclose(x, y, rtol=1e-12, atol=1e-12), name
