"""The gated RMSNorm oracle (oracle/gated_norm_f64.py) pinned on CPU: its forward against transformers'
Qwen3_5RMSNormGated (the module the reference's kernels replace) and against the reference's own float64
truth `ref_gated` restated (tests/test_layer.py:176-177 of the reference), its backward against float64 autograd."""
import pytest
import torch
import torch.nn.functional as F

from oracle import gated_norm_f64


def make(rows=37, d=128, seed=0):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, d, generator=gen, dtype=torch.float64)
    z = torch.randn(rows, d, generator=gen, dtype=torch.float64) * 2
    w = torch.randn(d, generator=gen, dtype=torch.float64) * 0.1 + 1.0
    return x, z, w


def test_forward_matches_transformers_module():
    """The module casts its input to float32 inside (its own rounding points), so the match is to float32 precision."""
    M = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
    x, z, w = make()
    m = M.Qwen3_5RMSNormGated(128, eps=gated_norm_f64.EPS).double()
    m.weight.data = w.clone()
    with torch.no_grad():
        ref = m(x, z)
    assert torch.allclose(gated_norm_f64.forward(x, z, w), ref, rtol=1e-5, atol=1e-6)


def test_forward_matches_the_float64_truth():
    x, z, w = make(rows=5, d=96, seed=1)
    ref = w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)) * F.silu(z)
    assert torch.allclose(gated_norm_f64.forward(x, z, w), ref, rtol=1e-14, atol=1e-15)


@pytest.mark.parametrize("d", [128, 1024, 36])
def test_backward_matches_float64_autograd(d):
    x, z, w = make(rows=11, d=d, seed=2)
    xs = [t.clone().requires_grad_(True) for t in (x, z, w)]
    o = xs[2] * (xs[0] * torch.rsqrt(xs[0].pow(2).mean(-1, keepdim=True) + 1e-6)) * F.silu(xs[1])
    do = torch.randn(o.shape, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    grads = torch.autograd.grad((o * do).sum(), xs)
    mine = gated_norm_f64.backward(x, z, w, do)
    for name, a, b in zip(("dx", "dz", "dw"), mine, grads):
        assert torch.allclose(a, b, rtol=1e-12, atol=1e-12), name
