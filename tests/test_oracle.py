"""The CPU oracle pinned against the reference's own outputs (tests/golden/*.npz, generated from the reference by
tests/golden/make_golden.py): the float64 recurrence, the chunked equations (forward and backward) and the drop-in
prologue against transformers' function. CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import gated_delta_f64 as ref
from oracle import parity

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F64 = torch.float64


def load(name):
    with np.load(os.path.join(GOLD, name)) as z:
        return {k: torch.from_numpy(z[k]) for k in z.files}


@pytest.mark.parametrize("name", ["recurrence_small.npz", "recurrence_stress.npz", "recurrence_strong_decay.npz"])
def test_recurrence_matches_reference(name):
    z = load(name)
    got = ref.recurrence_grads(z["q"], z["k"], z["v"], z["g"], z["beta"], z["s0"], z["do"], z["dsT"])
    for n, a in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), got):
        assert parity.rel_err(a, z[n]) < 1e-12, n


@pytest.mark.parametrize("name", ["recurrence_small.npz", "recurrence_stress.npz", "recurrence_strong_decay.npz"])
@pytest.mark.parametrize("C", [8, 16, 64])
def test_chunked_matches_reference_recurrence(name, C):
    """The chunked restatement (any chunk length, tail chunks) against the reference's float64 recurrence."""
    z = load(name)
    got = ref.chunked(z["q"], z["k"], z["v"], z["g"], z["beta"], z["s0"], z["do"], z["dsT"], C=C)
    tol = 1e-9 if "stress" in name else 1e-11
    for n, a in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), got):
        assert parity.rel_err(a, z[n]) < tol, (n, parity.rel_err(a, z[n]))


@pytest.mark.parametrize("name", ["chunk_eq_c8.npz", "chunk_eq_c64.npz"])
def test_chunked_matches_reference_checker(name):
    """Against tools/check_chunk_equations.py's own chunked(), on its own inputs ([T, D] layout, one head)."""
    z = load(name)
    C = int(z["C"])
    ex = lambda t: t[None, :, None]           # [T, D] -> [1, T, 1, D]; [T] -> [1, T, 1]
    got = ref.chunked(ex(z["q"]), ex(z["k"]), ex(z["v"]), ex(z["g"]), ex(z["beta"]), z["s0"][None, None],
                      ex(z["do"]), z["dsT"][None, None], C=C)
    want = [z[n] for n in ("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0")]
    for n, a, b in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), got, want):
        a = a.reshape(b.shape)
        assert (a - b).abs().max().item() < 1e-12, n


def test_dropin_matches_transformers_fp32():
    """The drop-in's float64 truth (l2 prologue, DK^-1/2 query scale, the rule, gradients of the raw inputs through the
    prologue) against transformers' fp32 function: within fp32 rounding."""
    z = load("transformers_fp32.npz")
    got = ref.dropin(z["q"], z["k"], z["v"], z["g"], z["beta"], z["s0"], z["do"], z["dsT"])
    for n, a in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), got):
        assert parity.rel_err(a, z[n]) < 2e-5, (n, parity.rel_err(a, z[n]))


def test_dropin_chunked_equals_recurrence():
    z = load("transformers_fp32.npz")
    a = ref.dropin(z["q"], z["k"], z["v"], z["g"], z["beta"], z["s0"], z["do"], z["dsT"], chunk=64)
    b = ref.dropin(z["q"], z["k"], z["v"], z["g"], z["beta"], z["s0"], z["do"], z["dsT"], chunk=None)
    for x, y in zip(a, b):
        assert parity.rel_err(x, y) < 1e-11


def test_reference_bf16_error_is_bf16_sized():
    """transformers on bf16 inputs runs its l2norm in bf16: its error against float64 is bf16-sized (this is the
    error the parity bar doubles). The fixture's outputs reproduce that error."""
    z = load("transformers_bf16.npz")
    bf = lambda t: t.to(torch.bfloat16)
    truth = ref.dropin(bf(z["q"]), bf(z["k"]), bf(z["v"]), z["g"], z["beta"], z["s0"], bf(z["do"]).float(), z["dsT"])
    errs = [parity.rel_err(z[n], t) for n, t in zip(("o", "sT", "dq", "dk", "dv", "dg", "dbeta", "ds0"), truth)]
    assert max(errs) < 5e-2 and min(errs) > 1e-5, errs


def test_gqa_dropin_sums_key_gradients():
    """GQA (value heads = 2 x key heads) equals the explicitly repeated call with the key-side gradients summed."""
    gen = torch.Generator().manual_seed(3)
    B, T, Hk, D = 1, 20, 2, 8
    q, k = torch.randn(B, T, Hk, D, generator=gen, dtype=F64), torch.randn(B, T, Hk, D, generator=gen, dtype=F64)
    v = torch.randn(B, T, 2 * Hk, D, generator=gen, dtype=F64)
    g, b = -torch.rand(B, T, 2 * Hk, generator=gen, dtype=F64), torch.rand(B, T, 2 * Hk, generator=gen, dtype=F64)
    do = torch.randn(B, T, 2 * Hk, D, generator=gen, dtype=F64)
    a = ref.dropin(q, k, v, g, b, do=do, chunk=8)
    r = ref.dropin(q.repeat_interleave(2, 2), k.repeat_interleave(2, 2), v, g, b, do=do, chunk=8)
    assert parity.rel_err(a[0], r[0]) < 1e-13
    assert parity.rel_err(a[2], r[2].view(B, T, Hk, 2, D).sum(3)) < 1e-13
    assert parity.rel_err(a[3], r[3].view(B, T, Hk, 2, D).sum(3)) < 1e-13


def test_identical_comparator():
    """The bit-identity comparator (tests/test_memory.py:37-46's): NaN-aware, sign of zero, dtype."""
    a = torch.tensor([0.0, float("nan"), 1.0])
    assert parity.identical(a, a.clone())
    assert not parity.identical(a, torch.tensor([-0.0, float("nan"), 1.0]))
    assert not parity.identical(a, a.double())


def test_packed_oracle_matches_the_recurrence_with_state_resets():
    """dropin_packed (each sequence run as its own row) against an independent restatement: one token recurrence over
    the whole packed stream that resets the state to s0[n] at each sequence's first token. Boundaries cover a
    one-token sequence, a chunk-exact one, an empty one and ragged tails."""
    gen = torch.Generator().manual_seed(7)
    T, H, D = 150, 2, 128
    cu = [0, 1, 65, 65, 129, 150]
    q, k, v = (torch.randn(1, T, H, D, generator=gen, dtype=torch.float64) for _ in range(3))
    g = -torch.rand(1, T, H, generator=gen, dtype=torch.float64) * 2
    beta = torch.rand(1, T, H, generator=gen, dtype=torch.float64)
    s0 = torch.randn(5, H, D, D, generator=gen, dtype=torch.float64) * 0.02
    o, sT = ref.dropin_packed(q, k, v, g, beta, cu, s0)
    qn, kn = ref.l2norm(q) * D ** -0.5, ref.l2norm(k)
    o2, sT2 = ref.recurrence_packed(qn, kn, v, g, beta, s0, cu)
    assert (o - o2).abs().max().item() < 1e-12 and (sT - sT2).abs().max().item() < 1e-12
    assert torch.equal(sT[2], s0[2])  # the empty sequence passes its state through
