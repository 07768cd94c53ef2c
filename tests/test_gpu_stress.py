"""The reference's numerical stress cases (tests/test_harness.py:19-31, :77-97 of the reference) run through the B200
kernels by the drop-in, forward + backward, every output and gradient against the float64 oracle with the north star's
bar (max error <= 2x transformers' own error against float64 on the same inputs, per tensor; oracle/parity.py):

- beta = 0 (no update) and beta = 1 - 1e-6, g = 0 (no decay) and g = -20 (strong decay), and both extremes at once;
- keys nearly parallel (each key a shared direction plus 10 % noise, adjacent k_i . k_j > 0.95: the chunk inverse's
  matrix I + L then has off-diagonal entries near beta, its hard case), with beta random / near 1 and g random / 0;
- a long sequence (T = 2048, one head);
- the committed float64 stress fixtures (tests/golden/recurrence_stress.npz: beta = 1 - 1e-6, g = 0, correlated
  keys; recurrence_strong_decay.npz: g = -20): their recipes at head width 128, and their own inputs zero-padded
  from their head widths to 128 (the l2 prologue leaves a zero-padded row's direction unchanged).

Inputs are built as the reference's make() builds them (q, k, v ~ N(0, 1), g = -U(0, 1), beta = U(0, 1),
s0 ~ N(0, 0.1)) and rounded to bf16 for q, k, v, dO; the rule normalises q and k itself (use_qk_l2norm_in_kernel).
Each case prints its per-tensor ratios (new error / transformers' error)."""
import os

import numpy as np
import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity, transformers_ref
from test_gpu_backward import NAMES, run_grads

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
D = 128


def make(B, T, H, seed=0, beta=None, g=None, corr=0.0):
    """The reference harness's fixture (tests/test_harness.py:19-31) for the drop-in: raw (not yet normalised) q, k in
    bf16, v in bf16, g / beta float32, s0 ~ N(0, 0.1); corr > 0 makes every key a shared direction plus (1 - corr)
    noise. Also dO (bf16) and dS_T cotangents."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=gen)
    k = torch.randn(B, T, H, D, generator=gen)
    if corr:
        k = corr * torch.randn(B, 1, H, D, generator=gen) + (1 - corr) * k
    v = torch.randn(B, T, H, D, generator=gen)
    gg = -torch.rand(B, T, H, generator=gen) if g is None else torch.full((B, T, H), float(g))
    bb = torch.rand(B, T, H, generator=gen) if beta is None else torch.full((B, T, H), float(beta))
    s0 = torch.randn(B, H, D, D, generator=gen) * 0.1
    do = torch.randn(B, T, H, D, generator=gen)
    dsT = torch.randn(B, H, D, D, generator=gen) * 0.1
    bf = torch.bfloat16
    return q.to(bf), k.to(bf), v.to(bf), gg, bb, s0, do.to(bf), dsT


def report(xs):
    q, k, v, g, beta, s0, do, dsT = xs
    got = run_grads(q, k, v, g, beta, s0, do, dsT)
    truth = ref.dropin(q, k, v, g, beta, s0, do.double(), dsT)
    theirs = transformers_ref.run(q, k, v, g, beta, s0, do=do, dsT=dsT)
    rep = parity.check(got, theirs, truth, names=NAMES)
    for name, t in zip(NAMES, got):
        assert t is None or bool(torch.isfinite(t.float()).all()), f"{name} has non-finite values"
    print({k_: round(v_["ratio"], 3) for k_, v_ in rep.items()})
    return rep


def ratios(rep):
    return {k_: round(v_["ratio"], 3) for k_, v_ in rep.items()}


@pytest.mark.parametrize("beta,g", [(0.0, None), (1.0 - 1e-6, None), (None, 0.0), (None, -20.0), (1.0 - 1e-6, 0.0)])
def test_stress(beta, g):
    """tests/test_harness.py:77-80 of the reference: B=1, T=48, H=2 there; here two chunks and a tail (T=150)."""
    rep = report(make(1, 150, 2, seed=0, beta=beta, g=g))
    assert not parity.failures(rep), ratios(rep)


@pytest.mark.parametrize("beta,g", [(None, None), (1.0 - 1e-6, 0.0), (1.0 - 1e-6, None)])
def test_correlated_keys(beta, g):
    """tests/test_harness.py:83-90 of the reference (corr 0.9, seed 6, T=96, H=2): adjacent normalised keys have
    k_i . k_j > 0.95."""
    xs = make(1, 96, 2, seed=6, beta=beta, g=g, corr=0.9)
    kn = ref.l2norm(xs[1].double())
    assert (kn[0, 1:, 0] * kn[0, :-1, 0]).sum(-1).min() > 0.95
    rep = report(xs)
    assert not parity.failures(rep), ratios(rep)


def test_long_sequence():
    """tests/test_harness.py:93-96 of the reference: B=1, T=2048, H=1."""
    rep = report(make(1, 2048, 1, seed=3))
    assert not parity.failures(rep), ratios(rep)


def _pad(x, n):
    """Zero-pad the last dimension to n."""
    return torch.nn.functional.pad(x, (0, n - x.shape[-1]))


@pytest.mark.parametrize("recipe", ["stress", "strong_decay"])
def test_fixture_recipes_at_full_width(recipe):
    """The committed stress fixtures' recipes (tests/golden/make_golden.py: the reference harness's make() with the
    same T, H, seed, beta, g and key correlation) at the kernels' head width 128."""
    if recipe == "stress":
        xs = make(1, 40, 1, seed=6, beta=1.0 - 1e-6, g=0.0, corr=0.9)
    else:
        xs = make(1, 70, 1, seed=2, g=-20.0)
    rep = report(xs)
    assert not parity.failures(rep), ratios(rep)


def golden_inputs(name):
    """A committed float64 fixture's inputs (q, k normalised already; the prologue renormalises the zero-padded rows
    to the same directions), zero-padded to D = 128, rounded to bf16."""
    with np.load(os.path.join(GOLD, name)) as z:
        f = {n: torch.from_numpy(z[n]) for n in z.files}
    bf = torch.bfloat16
    q, k, v = (_pad(f[n], D).to(bf) for n in ("q", "k", "v"))
    s0 = torch.zeros(1, f["s0"].shape[1], D, D, dtype=torch.float64)
    s0[:, :, :f["s0"].shape[2], :f["s0"].shape[3]] = f["s0"]
    dsT = torch.zeros_like(s0)
    dsT[:, :, :f["dsT"].shape[2], :f["dsT"].shape[3]] = f["dsT"]
    do = _pad(f["do"], D).to(bf)
    return q, k, v, f["g"].float(), f["beta"].float(), s0.float(), do, dsT.float()


def test_golden_strong_decay_inputs():
    """recurrence_strong_decay.npz (g = -20, D = 16) zero-padded to 128."""
    rep = report(golden_inputs("recurrence_strong_decay.npz"))
    assert not parity.failures(rep), ratios(rep)


def test_golden_stress_inputs():
    """recurrence_stress.npz (beta = 1 - 1e-6, g = 0, keys with k_i . k_j ~ 0.99, T = 40, D = 32) zero-padded to 128:
    the hardest case here. The per-chunk gradient's chain dA -> T1 = dA A^T -> dL = -A^T T1, A^T dVn and dVn V^T, and
    the reverse pass's W^T dVn cancel to a small fraction of their terms with nearly parallel keys at beta ~ 1 while
    transformers (fp32 on bf16-rounded inputs that are exact here) is unusually exact: every one of those operands is
    carried as bf16 hi + lo for this case to meet the bar."""
    rep = report(golden_inputs("recurrence_stress.npz"))
    assert not parity.failures(rep), ratios(rep)
