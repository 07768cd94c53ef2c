"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): parity metrics and the bar.

The bar (the float64 ground truth of tests/test_harness.py:34-57 in the reference): for every
output and gradient, max|new - f64| <= FACTOR * max|reference - f64|, the reference being transformers'
torch_chunk_gated_delta_rule run on the same inputs in their own dtypes (oracle/transformers_ref.py) and f64 the
float64 recompute (oracle/gated_delta_f64.py). A small absolute floor (ABS_FLOOR times the tensor's scale) keeps the
bar meaningful where the reference happens to be exact.
"""
from __future__ import annotations

import torch

FACTOR = 2.0
ABS_FLOOR = 1e-7
NAMES = ("o", "sT", "dquery", "dkey", "dvalue", "dg", "dbeta", "ds0")


def max_err(a, b) -> float:
    return (a.detach().cpu().double() - b.detach().cpu().double()).abs().max().item() if a.numel() else 0.0


def scale(b) -> float:
    return b.detach().abs().max().item() if b.numel() else 0.0


def rel_err(a, b) -> float:
    """max|a - b| / max|b|: the reference harness's metric (tests/test_harness.py:46,54)."""
    return max_err(a, b) / max(scale(b), 1e-12)


def check(new, ref, truth, names=NAMES, factor=FACTOR):
    """Per tensor: (new error, reference error, ratio, ok). `new`, `ref`, `truth` are sequences in `names` order; a
    None entry in `new` or `truth` is skipped."""
    report = {}
    for n, a, r, t in zip(names, new, ref, truth):
        if a is None or t is None:
            continue
        e_new = max_err(a, t)
        e_ref = max_err(r, t) if r is not None else 0.0
        bar = factor * e_ref + ABS_FLOOR * max(scale(t), 1.0)
        report[n] = dict(new=e_new, ref=e_ref, ratio=e_new / max(e_ref, 1e-30), ok=e_new <= bar)
    return report


def failures(report):
    return {k: v for k, v in report.items() if not v["ok"]}


def identical(a: torch.Tensor, b: torch.Tensor) -> bool:
    """NaN-aware exact equality plus equality of the raw bits (the reference's comparator, tests/test_memory.py:37-46)."""
    ints = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16,
            torch.float64: torch.int64}
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    na, nb = torch.isnan(a), torch.isnan(b)
    if not (torch.equal(na, nb) and torch.equal(a[~na], b[~nb])):
        return False
    return torch.equal(a.view(ints[a.dtype]), b.view(ints[b.dtype]))
