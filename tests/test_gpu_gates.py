"""The gates kernels (gd_gates_fwd / gd_gates_bwd through macai_b200.gates) against the float64 oracle, with the
north star's bar: max error <= 2x that of the PyTorch expression the reference replaces (run on the CPU in the inputs'
dtypes, float32 math: transformers' Qwen3.5 gates), plus a small absolute floor for exactly representable results."""
import pytest
import torch
import torch.nn.functional as F

from oracle import gates_f64, parity

pytestmark = pytest.mark.gpu


def make(shape, dtype, wdtype=torch.float32, seed=0):
    gen = torch.Generator().manual_seed(seed)
    H = shape[-1]
    b = (torch.randn(shape, generator=gen) * 3).to(dtype)
    a = (torch.randn(shape, generator=gen) * 8).to(dtype)  # a + dt_bias crosses the softplus threshold of 20
    A_log = torch.log(torch.empty(H).uniform_(1, 16, generator=gen)).to(wdtype)
    dt_bias = (torch.randn(H, generator=gen) * 4).to(wdtype)
    return b, a, A_log, dt_bias


def torch_gates(b, a, A_log, dt_bias):
    """The expression the reference's kernels replace, in float32 (transformers' layer)."""
    beta = b.float().sigmoid()
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return beta, g


def within_bar(got, theirs, truth, name):
    e_got, e_theirs = parity.max_err(got, truth), parity.max_err(theirs, truth)
    floor = parity.ABS_FLOOR * max(parity.scale(truth), 1.0)
    assert e_got <= 2.0 * e_theirs + floor, (name, e_got, e_theirs)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(2, 100, 16), (1, 37, 300), (4, 1024, 32)])
def test_forward_parity(dtype, shape):
    from macai_b200.gates import gates
    x = make(shape, dtype, seed=shape[1])
    beta, g = gates(*(t.cuda() for t in x))
    truth = gates_f64.forward(*x)
    theirs = torch_gates(*x)
    assert beta.dtype == torch.float32 and g.dtype == torch.float32 and beta.shape == x[0].shape
    within_bar(beta.cpu(), theirs[0], truth[0], "beta")
    within_bar(g.cpu(), theirs[1], truth[1], "g")


@pytest.mark.parametrize("dtype,wdtype", [(torch.bfloat16, torch.float32), (torch.float32, torch.float32),
                                          (torch.bfloat16, torch.bfloat16)])
def test_backward_parity(dtype, wdtype):
    from macai_b200.gates import gates
    x = make((2, 200, 16), dtype, wdtype, seed=3)
    gen = torch.Generator().manual_seed(4)
    dbeta = torch.randn(x[0].shape, generator=gen)
    dg = torch.randn(x[0].shape, generator=gen)
    xs = [t.cuda().requires_grad_(True) for t in x]
    beta, g = gates(*xs)
    ((beta * dbeta.cuda()).sum() + (g * dg.cuda()).sum()).backward()
    got = [t.grad.cpu() for t in xs]
    xt = [t.clone().requires_grad_(True) for t in x]
    tb, tg = torch_gates(*xt)
    ((tb * dbeta).sum() + (tg * dg).sum()).backward()
    theirs = [t.grad for t in xt]
    truth = gates_f64.backward(*x, dbeta, dg)
    for name, gt, th, tr, xin in zip(("db", "da", "dA_log", "ddt_bias"), got, theirs, truth, x):
        assert gt.dtype == xin.dtype
        within_bar(gt, th, tr, name)


def test_missing_cotangent_and_frozen_weights():
    """Only g used (dbeta is None: db is zero); A_log and dt_bias frozen (no per-head sums), as in LoRA training."""
    from macai_b200.gates import gates
    b, a, A_log, dt_bias = (t.cuda() for t in make((1, 64, 8), torch.bfloat16, seed=5))
    b.requires_grad_(True)
    a.requires_grad_(True)
    beta, g = gates(b, a, A_log, dt_bias)
    g.sum().backward()
    assert torch.count_nonzero(b.grad) == 0
    _, da, _, _ = gates_f64.backward(b.detach().cpu(), a.detach().cpu(), A_log.cpu(), dt_bias.cpu(),
                                     torch.zeros(b.shape), torch.ones(b.shape))
    assert torch.allclose(a.grad.float().cpu(), da.float(), rtol=1e-2, atol=1e-6)


def test_per_head_sums_are_deterministic():
    from macai_b200.gates import gates
    x = make((8, 1000, 24), torch.bfloat16, seed=6)
    runs = []
    for _ in range(3):
        xs = [t.cuda().requires_grad_(True) for t in x]
        beta, g = gates(*xs)
        (beta.sum() + (g * 0.5).sum()).backward()
        runs.append([t.grad.cpu() for t in xs])
    for r in runs[1:]:
        for u, v in zip(runs[0], r):
            assert parity.identical(u, v)
