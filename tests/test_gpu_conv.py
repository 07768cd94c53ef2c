"""The convolution-path kernels (gd_conv_fwd / gd_conv_bwd through macai_b200.conv) with the reference's own protocol
for this part (tests/test_layer.py:33-99, :221-268 of the reference): inputs drawn exactly representable in the run's
dtype, the real widths of Qwen3.5-0.8B and 9B (the 9B one with two value heads a key head), odd token counts, and for
q, k, v and every needed gradient the relative error against float64 (max|a - f64| / max|f64|) at most twice that of
transformers' own path (its PyTorch fallback: conv1d over the channel-first transpose, SiLU, split, reshape,
repeat_interleave), run here on the same GPU in the same dtype, plus one float32 ulp of the scale as a floor."""
import pytest
import torch
import torch.nn.functional as F

from oracle import conv_f64

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
DT = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}
LIN = {"0.8b": dict(kd=2048, vd=2048, dk=128, rep=1, dv=128), "9b": dict(kd=2048, vd=4096, dk=128, rep=2, dv=128)}
ULP = 2.0 ** -23


def draw(shape, dtype, scale=1.0, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=gen, dtype=torch.float64) * scale).to(dtype).double()


def rel(a, r):
    return ((a.double() - r).abs().max() / r.abs().max().clamp_min(1e-300)).item()


def layout(y, c, B, T):
    q, k, v = torch.split(y, [c["kd"], c["kd"], c["vd"]], dim=-1)
    q = q.reshape(B, T, -1, c["dk"]).repeat_interleave(c["rep"], dim=2)
    k = k.reshape(B, T, -1, c["dk"]).repeat_interleave(c["rep"], dim=2)
    return q, k, v.reshape(B, T, -1, c["dv"])


def run(fn, x, w, dtype, trained, gouts):
    xl = x.to("cuda", dtype).requires_grad_(True)
    wl = w.to("cuda", dtype).requires_grad_(trained)
    outs = fn(xl, wl)
    torch.autograd.backward(outs, [g.to("cuda", o.dtype) for g, o in zip(gouts, outs)])
    return ([o.detach().cpu().double() for o in outs], xl.grad.detach().cpu().double(),
            wl.grad.detach().cpu().double() if trained else None)


def check(model, B, T, dtype, trained, seed=11):
    c = LIN[model]
    C = 2 * c["kd"] + c["vd"]
    x = draw((B, T, C), dtype, seed=seed)
    w = draw((C, 1, 4), dtype, scale=0.3, seed=seed + 1)
    args = (c["kd"], c["dk"], c["rep"], c["dv"])
    ro = conv_f64.forward(x, w, *args)
    gouts = [draw(o.shape, dtype, seed=100 + i) for i, o in enumerate(ro)]
    rdx, rdw = conv_f64.backward(x, w, *gouts, *args)

    def torch_path(x_, w_):
        return layout(F.silu(F.conv1d(x_.transpose(1, 2), w_, padding=3, groups=C)[:, :, :T]).transpose(1, 2), c, B, T)

    def fused(x_, w_):
        from macai_b200.conv import conv_qkv
        return conv_qkv(x_, w_, *args)
    to, tdx, tdw = run(torch_path, x, w, dtype, trained, gouts)
    fo, fdx, fdw = run(fused, x, w, dtype, trained, gouts)
    rows = {n: (rel(t, r), rel(f, r)) for n, t, f, r in zip("qkv", to, fo, ro)}
    rows["dx"] = (rel(tdx, rdx), rel(fdx, rdx))
    if trained:
        rows["dw"] = (rel(tdw.reshape(-1, 4), rdw), rel(fdw.reshape(-1, 4), rdw))
    bad = {k: v for k, v in rows.items() if not v[1] <= 2 * v[0] + ULP}
    assert not bad, f"fused error over twice transformers' (transformers, fused): {bad}"


@pytest.mark.parametrize("dtype", DTYPES, ids=DT.get)
@pytest.mark.parametrize("bt", [(1, 1), (2, 3), (2, 33), (3, 100)], ids=str)
@pytest.mark.parametrize("model", ["0.8b", "9b"])
def test_conv_path(model, bt, dtype):
    check(model, *bt, dtype, False)


@pytest.mark.parametrize("dtype", DTYPES, ids=DT.get)
@pytest.mark.parametrize("model", ["0.8b", "9b"])
def test_conv_path_trained_weight(model, dtype):
    """The weight's gradient when it trains (fixed-order partial rows, then a tree sum)."""
    check(model, 2, 33, dtype, True)


def test_many_tiles_weight_gradient():
    """More (row, time tile) pairs than partial rows (256; 64-step tiles at this size): each row block walks several
    tiles. The short cases above run 16-step tiles."""
    check("0.8b", 8, 2100, torch.bfloat16, True, seed=21)


def test_output_dtypes_and_zero_cotangents():
    from macai_b200.conv import conv_qkv
    c = LIN["9b"]
    C = 2 * c["kd"] + c["vd"]
    x = torch.randn(2, 40, C, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(C, 1, 4, device="cuda") * 0.3).to(torch.bfloat16).requires_grad_(True)
    q, k, v = conv_qkv(x, w, c["kd"], c["dk"], c["rep"], c["dv"])
    assert q.dtype == k.dtype == torch.bfloat16 and v.dtype == torch.float32
    assert q.shape == (2, 40, 32, 128) and v.shape == (2, 40, 32, 128)
    v.sum().backward()  # q and k unused: their cotangents are None (zero)
    _, rdw = conv_f64.backward(x.detach().cpu(), w.detach().cpu(), None, None, torch.ones(v.shape), c["kd"], c["dk"],
                               c["rep"], c["dv"])
    assert torch.count_nonzero(x.grad[..., :2 * c["kd"]]) == 0
    assert torch.allclose(w.grad.float().reshape(-1, 4).cpu().double(), rdw, rtol=2e-2, atol=1e-3)


def test_weight_gradient_is_deterministic():
    from macai_b200.conv import conv_qkv
    c = LIN["0.8b"]
    C = 2 * c["kd"] + c["vd"]
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4, 700, C, device="cuda", generator=gen).to(torch.bfloat16)
    w0 = (torch.randn(C, 1, 4, device="cuda", generator=gen) * 0.3).to(torch.bfloat16)
    grads = []
    for _ in range(3):
        w = w0.clone().requires_grad_(True)
        q, k, v = conv_qkv(x, w, c["kd"], c["dk"], c["rep"], c["dv"])
        (q.float().sum() + k.float().square().sum() + v.sum()).backward()
        grads.append(w.grad.clone())
    assert all(torch.equal(grads[0], g) for g in grads[1:])
