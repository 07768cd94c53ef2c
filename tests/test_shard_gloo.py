"""The multi-GPU layer's host logic on CPU ranks (gloo, world size 2): partition by batch rows or key-head groups,
each rank computes its slice (here with the float64 oracle standing in for the GPU kernels), gather, and the result is
bit-identical to the unsharded computation, gradients included. Also: a rank that never joins makes the others fail
with an error (process-group timeout), not hang."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from macai_b200.gated_delta import shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(B, T, Hk, H, D=8, seed=0):
    gen = torch.Generator().manual_seed(seed)
    f = torch.float64
    q, k = torch.randn(B, T, Hk, D, generator=gen, dtype=f), torch.randn(B, T, Hk, D, generator=gen, dtype=f)
    v = torch.randn(B, T, H, D, generator=gen, dtype=f)
    g, b = -torch.rand(B, T, H, generator=gen, dtype=f), torch.rand(B, T, H, generator=gen, dtype=f)
    s0 = torch.randn(B, H, D, D, generator=gen, dtype=f) * 0.1
    do = torch.randn(B, T, H, D, generator=gen, dtype=f)
    dsT = torch.randn(B, H, D, D, generator=gen, dtype=f) * 0.1
    return q, k, v, g, b, s0, do, dsT


def _worker(rank, world, port, shape, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import gated_delta_f64 as ref
        B, T, Hk, H = shape
        full = _inputs(B, T, Hk, H)
        s = shard.partition(B, H, Hk, world, rank)
        loc = shard.take(s, *full)
        res = ref.dropin(*loc[:6], do=loc[6], dsT=loc[7], chunk=8)
        kinds = ["bth", "bh", "bth", "bth", "bth", "bth", "bth", "bh"]
        got = [shard.gather(s, x, kd) for x, kd in zip(res, kinds)]
        if rank == 0:
            want = ref.dropin(*full[:6], do=full[6], dsT=full[7], chunk=8)
            out.put([bool(torch.equal(a, b)) for a, b in zip(got, want)])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape", [(4, 20, 2, 2), (1, 20, 4, 8)])  # batch-row split; key-head split with GQA
def test_sharded_equals_unsharded(shape):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert all(res), res
    assert all(p.exitcode == 0 for p in procs)


def test_partition_rules():
    s = shard.partition(64, 32, 32, 8, 3)
    assert (s.b0, s.b1, s.h0, s.h1, s.dim) == (24, 32, 0, 32, 0)
    s = shard.partition(1, 32, 32, 8, 7)
    assert (s.b0, s.b1, s.h0, s.h1, s.dim) == (0, 1, 28, 32, 2)
    s = shard.partition(2, 32, 16, 4, 1)           # GQA, key heads 4-7 serve value heads 8-15
    assert (s.b0, s.b1, s.hk0, s.hk1, s.h0, s.h1) == (0, 2, 4, 8, 8, 16)
    with pytest.raises(ValueError):
        shard.partition(3, 6, 3, 2, 0)


def _late_worker(rank, world, port, out):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        t = torch.ones(1)
        dist.all_reduce(t)
        out.put(("ok", rank))
    except Exception as e:  # the peer never joins: the rendezvous or the collective times out with an error
        out.put(("error", type(e).__name__))


def test_missing_rank_times_out_with_error():
    """Rank 1 never starts: rank 0's process group must end in an exception within its timeout, not hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_late_worker, args=(0, 2, _port(), q))
    p.start()
    kind, _ = q.get(timeout=120)
    p.join(timeout=30)
    assert kind == "error"
