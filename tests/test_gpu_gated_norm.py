"""The gated RMSNorm kernels (gd_gnorm_fwd / gd_gnorm_bwd through macai_b200.gated_norm) with the reference's own
protocol for this part (tests/test_layer.py:33-99, :176-217 of the reference): inputs drawn exactly representable in
the run's dtype, the real widths of Qwen3.5-0.8B and 9B (16 / 32 value heads of 128), odd token counts, and for o and
every needed gradient the relative error against float64 (max|a - f64| / max|f64|) at most twice that of transformers'
own module (Qwen3_5RMSNormGated, run here on the same GPU in the same dtype), plus one float32 ulp of the scale as a
floor for results the module happens to get exact."""
import pytest
import torch

from oracle import gated_norm_f64

pytestmark = pytest.mark.gpu

M = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
DT = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}
HV = {"0.8b": 16, "9b": 32}
SHAPES = [(1, 1), (2, 7), (3, 33), (2, 129)]
EPS = 1e-6
ULP = 2.0 ** -23


def draw(shape, dtype, scale=1.0, seed=0, shift=0.0):
    """float64 values exactly representable in dtype."""
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=gen, dtype=torch.float64) * scale + shift).to(dtype).double()


def rel(a, r):
    return ((a.double() - r).abs().max() / r.abs().max().clamp_min(1e-300)).item()


def run(fn, xs, dtypes, needs, gout, device):
    leaves = [x.detach().to(device, d).clone().requires_grad_(n) for x, d, n in zip(xs, dtypes, needs)]
    o = fn(*leaves)
    o.backward(gout.to(device, o.dtype))
    return o.detach().cpu().double(), [x.grad.detach().cpu().double() if n else None for x, n in zip(leaves, needs)]


def transformers_path(d):
    def fn(x, z, w):
        m = M.Qwen3_5RMSNormGated(d, eps=EPS).to(x.device)
        return torch.func.functional_call(m, {"weight": w}, (x, z))
    return fn


def fused(x, z, w):
    from macai_b200.gated_norm import gated_rms_norm
    return gated_rms_norm(x, z, w, EPS)


def check(rows, d, dtype, trained, wdtype=None, seed=8):
    x = draw((rows, d), dtype, seed=seed)
    z = draw((rows, d), dtype, seed=seed + 1)
    w = draw((d,), wdtype or dtype, scale=0.1, seed=seed + 2, shift=1.0)
    gout = draw((rows, d), dtype, seed=100)
    needs = [True, True, trained]
    ro = gated_norm_f64.forward(x, z, w, EPS)
    rg = gated_norm_f64.backward(x, z, w, gout, EPS)
    dtypes = [dtype, dtype, wdtype or dtype]
    to, tg = run(transformers_path(d), [x, z, w], dtypes, needs, gout, "cuda")
    fo, fg = run(fused, [x, z, w], dtypes, needs, gout, "cuda")
    rows_ = {"o": (rel(to, ro), rel(fo, ro))}
    for name, r, t, f, n in zip(("dx", "dz", "dw"), rg, tg, fg, needs):
        if n:
            rows_[name] = (rel(t, r), rel(f, r))
    bad = {k: v for k, v in rows_.items() if not v[1] <= 2 * v[0] + ULP}
    assert not bad, f"fused error over twice transformers' (transformers, fused): {bad}"
    return rows_


@pytest.mark.parametrize("dtype", DTYPES, ids=DT.get)
@pytest.mark.parametrize("bt", SHAPES, ids=str)
@pytest.mark.parametrize("model", ["0.8b", "9b"])
def test_gated_norm(model, bt, dtype):
    check(bt[0] * bt[1] * HV[model], 128, dtype, False)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT.get)
@pytest.mark.parametrize("model", ["0.8b", "9b"])
def test_gated_norm_trained_weight(model, dtype):
    """The weight's gradient when the weight trains (fixed-order partial rows, then a second pass)."""
    check(3 * 33 * HV[model], 128, dtype, True)


@pytest.mark.parametrize("d", [96, 256, 1024])
def test_other_widths_and_float32_weight(d):
    """Widths off the 128-column grid and above it, with a float32 weight under bf16 activations (h not rounded)."""
    check(300, d, torch.bfloat16, True, wdtype=torch.float32, seed=20)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT.get)
@pytest.mark.parametrize("d", [4, 20, 100, 520])
def test_team_shapes(d, dtype):
    """Every row-team shape of the generic kernels: one lane a row (d = 4), teams of 8 and 32 lanes with 8-byte chunks
    at 16 bits (20, 100: not multiples of 8), and 32-lane teams holding several chunks each with the last ones past
    the row (520), trained weight included."""
    check(257, d, dtype, True, seed=50 + d)


def test_large_rows_weight_gradient():
    """More rows than the backward's partial rows (1024 CTAs): every CTA sums several rows per warp."""
    check(70_000, 128, torch.bfloat16, True, seed=30)


def test_weight_gradient_is_deterministic():
    from macai_b200.gated_norm import gated_rms_norm
    x = draw((50_000, 128), torch.bfloat16, seed=40).to("cuda", torch.bfloat16)
    z = draw((50_000, 128), torch.bfloat16, seed=41).to("cuda", torch.bfloat16)
    w0 = draw((128,), torch.bfloat16, seed=42).to("cuda", torch.bfloat16)
    grads = []
    for _ in range(3):
        w = w0.clone().requires_grad_(True)
        gated_rms_norm(x, z, w, EPS).float().square().sum().backward()
        grads.append(w.grad.clone())
    assert all(torch.equal(grads[0], g) for g in grads[1:])


def test_empty_rows():
    from macai_b200.gated_norm import gated_rms_norm
    x = torch.empty(0, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    z = torch.empty(0, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    o = gated_rms_norm(x, z, w, EPS)
    o.sum().backward()
    assert o.shape == (0, 128) and torch.count_nonzero(w.grad) == 0
