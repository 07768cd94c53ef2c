"""Sharding the rule over GPUs by independent (batch row, head) slices.

Every (batch row, value head) of the gated delta rule is independent in the forward and in the backward: the only
cross-head coupling is the sum of the query/key gradients over the value heads one key head serves, which stays inside
a slice because slices are cut on key-head boundaries. A rank computes its slice with no communication; results are
gathered (torch.distributed all_gather, NCCL on GPUs) only where a caller needs the whole tensor, e.g. the final
states of a long prefill sharded over heads.

The reference runs on one device and has no counterpart; this module is the multi-GPU layer of the B200 build.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Slice:
    """Batch rows [b0, b1) and value heads [h0, h1) (key heads [hk0, hk1)) of one rank."""
    b0: int
    b1: int
    h0: int
    h1: int
    hk0: int
    hk1: int
    dim: int  # the dimension the ranks split: 0 = batch rows, 2 = heads


def partition(B: int, H: int, HK: int, world: int, rank: int) -> Slice:
    """Contiguous, equal slices: batch rows when B divides evenly over the ranks, else key-head groups (with their
    value heads). Raises ValueError when neither divides."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if B % world == 0:
        n = B // world
        return Slice(rank * n, (rank + 1) * n, 0, H, 0, HK, 0)
    if HK % world == 0:
        nk = HK // world
        rep = H // HK
        return Slice(0, B, rank * nk * rep, (rank + 1) * nk * rep, rank * nk, (rank + 1) * nk, 2)
    raise ValueError(f"neither the batch ({B}) nor the key heads ({HK}) divide over {world} ranks")


def take(s: Slice, q, k, v, g, beta, s0=None, do=None, dsT=None):
    """This rank's contiguous inputs ([B, T, H, ...] tensors sliced on batch rows or heads; states on [B, H])."""
    def bth(x, heads_k=False):
        if x is None:
            return None
        h0, h1 = (s.hk0, s.hk1) if heads_k else (s.h0, s.h1)
        return x[s.b0:s.b1, :, h0:h1].contiguous()

    def bh(x):
        return None if x is None else x[s.b0:s.b1, s.h0:s.h1].contiguous()

    return (bth(q, True), bth(k, True), bth(v), bth(g), bth(beta), bh(s0), bth(do), bh(dsT))


def gather(s: Slice, local: torch.Tensor, kind: str, group=None) -> torch.Tensor:
    """All ranks' slices of one result, concatenated: kind "bth" ([B, T, H, ...]) or "bh" ([B, H, ...])."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    if s.dim == 0:
        return torch.cat(parts, 0)
    return torch.cat(parts, 2 if kind == "bth" else 1)
