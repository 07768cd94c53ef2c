"""Generates the golden fixtures in this directory from the reference itself (run in the build container, where the
reference checkout and transformers are importable):

    python tests/golden/make_golden.py /path/to/reference

- recurrence_*.npz: the reference's float64 ground truth, macai.gated_delta.recurrent_reference
  (src/macai/gated_delta/op.py:301-314), with input gradients by float64 autograd and the harness's seeded cotangents
  (tests/test_harness.py:19-57, make() and check()).
- chunk_eq_*.npz: the reference's own float64 chunked forward/backward checker, tools/check_chunk_equations.py:22-79
  (`chunked`), on its own seeded inputs (:81-88) and on a C=64 case.
- transformers_*.npz: transformers' torch_chunk_gated_delta_rule (the function the drop-in replaces), fp32 and bf16, with
  gradients, on the inputs of the reference's transformers-parity test (tests/test_gated_delta.py:37-56) at a reduced
  head width.

Nothing at test time reads the reference checkout; the tests read only these .npz files.
"""
import os
import runpy
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def save(name, **arrays):
    out = {}
    for k, v in arrays.items():
        if v is None:
            continue
        t = v.detach().cpu()
        if t.dtype == torch.bfloat16:
            t = t.float()                       # bf16 values are exact in fp32; the test casts back
        out[k] = t.numpy()
    np.savez_compressed(os.path.join(HERE, name), **out)
    print(name, sum(a.nbytes for a in out.values()), "bytes raw")


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from macai.gated_delta import l2norm, recurrent_reference           # noqa: E402  (reference package)

    def make(B, T, H, DK, DV, seed=0, beta=None, g=None, state=True, corr=0.0):
        # tests/test_harness.py:19-31, restated (the reference's fixture)
        gen = torch.Generator().manual_seed(seed)
        q = l2norm(torch.randn(B, T, H, DK, generator=gen, dtype=torch.float64)) * DK ** -0.5
        k = torch.randn(B, T, H, DK, generator=gen, dtype=torch.float64)
        if corr:
            k = corr * torch.randn(B, 1, H, DK, generator=gen, dtype=torch.float64) + (1 - corr) * k
        k = l2norm(k)
        v = torch.randn(B, T, H, DV, generator=gen, dtype=torch.float64)
        gg = (-torch.rand(B, T, H, generator=gen, dtype=torch.float64)) if g is None else torch.full((B, T, H), float(g), dtype=torch.float64)
        bb = torch.rand(B, T, H, generator=gen, dtype=torch.float64) if beta is None else torch.full((B, T, H), float(beta), dtype=torch.float64)
        s0 = (torch.randn(B, H, DK, DV, generator=gen, dtype=torch.float64) * 0.1) if state else torch.zeros(B, H, DK, DV, dtype=torch.float64)
        return q, k, v, gg, bb, s0

    def recurrence_case(name, xs):
        leaves = [x.clone().requires_grad_(True) for x in xs]
        o, sT = recurrent_reference(*leaves)
        gen = torch.Generator().manual_seed(9)
        w_o = torch.randn(o.shape, generator=gen, dtype=torch.float64)
        w_s = torch.randn(sT.shape, generator=gen, dtype=torch.float64)
        ((o * w_o).sum() + (sT * w_s).sum()).backward()
        save(name, q=xs[0], k=xs[1], v=xs[2], g=xs[3], beta=xs[4], s0=xs[5], do=w_o, dsT=w_s, o=o, sT=sT,
             dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad, dg=leaves[3].grad, dbeta=leaves[4].grad,
             ds0=leaves[5].grad)

    recurrence_case("recurrence_small.npz", make(1, 37, 2, 32, 16, seed=0))
    recurrence_case("recurrence_stress.npz", make(1, 40, 1, 32, 16, seed=6, beta=1.0 - 1e-6, g=0.0, corr=0.9))
    recurrence_case("recurrence_strong_decay.npz", make(1, 70, 1, 16, 16, seed=2, g=-20.0))

    # the reference's chunked checker, executed from its file with its own globals
    mod = runpy.run_path(os.path.join(ref_root, "tools", "check_chunk_equations.py"), run_name="golden")
    chunked = mod["chunked"]
    for name, (T, C, DK, DV, seed) in {"chunk_eq_c8.npz": (21, 8, 6, 5, 0), "chunk_eq_c64.npz": (100, 64, 16, 8, 1)}.items():
        chunked.__globals__.update(T=T, C=C, DK=DK, DV=DV)
        gen = torch.Generator().manual_seed(seed)
        dt = torch.float64
        q = torch.nn.functional.normalize(torch.randn(T, DK, generator=gen, dtype=dt), dim=-1) * DK ** -0.5
        k = torch.nn.functional.normalize(torch.randn(T, DK, generator=gen, dtype=dt), dim=-1)
        v = torch.randn(T, DV, generator=gen, dtype=dt)
        g = -torch.rand(T, generator=gen, dtype=dt) * 2.0
        b = torch.rand(T, generator=gen, dtype=dt)
        S0 = torch.randn(DK, DV, generator=gen, dtype=dt)
        dO = torch.randn(T, DV, generator=gen, dtype=dt)
        dS = torch.randn(DK, DV, generator=gen, dtype=dt)
        O, S, (dq, dk, dv, dg, db, ds0) = chunked(q, k, v, g, b, S0, dO, dS)
        save(name, C=torch.tensor(C), q=q, k=k, v=v, g=g, beta=b, s0=S0, do=dO, dsT=dS, o=O, sT=S, dq=dq, dk=dk,
             dv=dv, dg=dg, dbeta=db, ds0=ds0)

    # transformers' function (third-party; the drop-in's own parity target, tests/test_gated_delta.py:37-56)
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_chunk_gated_delta_rule as tf_rule
    for dtype, name in ((torch.float32, "transformers_fp32.npz"), (torch.bfloat16, "transformers_bf16.npz")):
        gen = torch.Generator().manual_seed(1)
        B, T, H, DK, DV = 1, 100, 2, 32, 32
        q = torch.randn(B, T, H, DK, generator=gen).to(dtype).requires_grad_(True)
        k = torch.randn(B, T, H, DK, generator=gen).to(dtype).requires_grad_(True)
        v = torch.randn(B, T, H, DV, generator=gen).to(dtype).requires_grad_(True)
        g = (-torch.rand(B, T, H, generator=gen)).requires_grad_(True)
        beta = torch.rand(B, T, H, generator=gen).requires_grad_(True)
        s0 = (torch.randn(B, H, DK, DV, generator=gen) * 0.1).requires_grad_(True)
        do = torch.randn(B, T, H, DV, generator=gen)
        dsT = torch.randn(B, H, DK, DV, generator=gen)
        o, sT = tf_rule(q, k, v, g, beta, chunk_size=64, initial_state=s0, output_final_state=True,
                        use_qk_l2norm_in_kernel=True)
        ((o.float() * do).sum() + (sT * dsT).sum()).backward()
        save(name, q=q, k=k, v=v, g=g, beta=beta, s0=s0, do=do, dsT=dsT, o=o, sT=sT, dq=q.grad, dk=k.grad,
             dv=v.grad, dg=g.grad, dbeta=beta.grad, ds0=s0.grad)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
