"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the chunked gated delta rule.

Nothing in the product package imports this directory. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` use it, as the checker and the timed CPU baseline.

Modules:
- `gated_delta_f64`: float64 restatements of the reference's recurrence (src/macai/gated_delta/op.py:301-314), its
  l2 prologue (src/macai/gated_delta/_norm.py:1-9) and its chunked forward/backward equations
  (tools/check_chunk_equations.py:22-79), pinned against golden vectors in tests/golden/.
- `transformers_ref`: the third-party "reference torch implementation" (transformers' torch_chunk_gated_delta_rule,
  pinned 5.22.1 by the reference's requirements.txt:4, 5.5.0 installed here) run on the CPU, used for the parity bar
  (2x its own error against float64) and as the timed CPU baseline.
- `parity`: the error metrics and the bar.
- `gates_f64`, `gated_norm_f64`: float64 restatements of the layer steps either side of the rule (the gates before
  it, src/macai/layer/_gates.py; the gated RMSNorm after it, src/macai/layer/_gated_norm.py), pinned on the CPU
  against float64 autograd of the PyTorch expressions they replace.
"""
