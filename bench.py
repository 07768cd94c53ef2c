"""Benchmark of the chunked gated delta rule, forward + backward, on B200 (sm_100a).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1|2|3|4] [--impl b200|reference]

One step = the forward (o, S_T) and the backward (dq, dk, dv, dg, dbeta, ds0; chunk states recomputed) of one batch of
the configuration through the library's C ABI (include/gated_delta_b200.h: gd_forward + gd_backward), captured once in
a CUDA graph. The headline metric: tokens/s (tokens = B * T) for forward + backward at config 1 (B=4, T=1024, H=16,
dk=dv=128, bf16, chunk 64, l2-normalised q/k). Inputs are seeded synthetic tensors: q, k, v ~ N(0, 1),
beta = sigmoid(N(0, 1)), g = -exp(U(log 1, log 16)) * softplus(N(0, 1)), dO ~ N(0, 1).

Multi-GPU (torchrun, one process per GPU): the headline is weak scaling over independent (batch, head) slices. Every
rank owns config 1's B batch rows of a global batch of N * B rows; there is no collective on the data path. The time
is the maximum over ranks of the device time (CUDA events), taken with an NCCL all-reduce(max) after the timed region.
Two sharded legs ride along (keys "c3" and "c4"; also at N = 1, as their one-GPU points):
  c4  B=64, T=4096, H=32 forward + backward, batch rows split over the ranks (64 / N each; strong scaling), plus a
      bit-identity check: one row of every rank's gradients, gathered (NCCL), against the same rows computed in one
      call on rank 0's GPU;
  c3  B=1, T=32768, H=32 forward, heads split over the ranks (32 / N each; strong scaling), the final states gathered
      by NCCL all_gather_into_tensor inside the timed region.

Printed (rank 0), one JSON line:
  value        whole-job tokens/s with inputs resident in HBM (sum of per-step device times; L2 flushed between steps)
  e2e          the same metric with every step's inputs copied host->device from pinned memory and every output copied
               back, inside the timed region (a CPU caller's view of the C ABI); steps overlap as in an input pipeline
               (next inputs in and previous outputs out on two copy streams while a step computes)
  roofline     the dominant kernel's achieved rate against MEASURED_PEAKS.json (per-kernel CUDA-event timing pass)
  cpu_baseline transformers' torch_chunk_gated_delta_rule (the reference torch implementation; oracle/transformers_ref.py)
               forward + backward on a bounded sample on this host's cores (rank 0, N = 1 only)
--impl reference runs only that CPU implementation (all host threads) and prints its line.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mac-ai-engineering_b200"))
sys.path.insert(0, ROOT)

METRIC = "gated-delta fwd+bwd tokens/s (B4 T1024 H16 d128 bf16)"
# the reference's own published number for this shape and pass (Apple M3 Max, Metal; not re-measurable here): 10.210 ms fwd+bwd at B4 T1024 H16 -> 401,175 tokens/s (docs/series_layer.md:1679-1684 of the reference)
PUBLISHED_TOKENS_S = 4 * 1024 / 10.210e-3
CONFIGS = {
    # B, T, H value heads, HK key heads, D; s0: an initial state (and its gradient); final: the final state is
    # returned (output_final_state); forward only. Config 1 is called as the reference's benchmark calls it
    # (bench/bench_gated_delta.py:64-83: the output only, no initial or final state).
    1: dict(B=4, T=1024, H=16, HK=16, D=128, s0=False, final=False, fwd_only=False,
            tag="c1: B4 T1024 H16 d128 fwd+bwd"),
    2: dict(B=2, T=1024, H=32, HK=16, D=128, s0=True, final=True, fwd_only=False,
            tag="c2: B2 T1024 Hk16 Hv32 d128 fwd+bwd, s0"),
    3: dict(B=1, T=32768, H=32, HK=32, D=128, s0=False, final=True, fwd_only=True,
            tag="c3: B1 T32768 H32 d128 forward"),
    4: dict(B=64, T=4096, H=32, HK=32, D=128, s0=False, final=False, fwd_only=False,
            tag="c4: B64 T4096 H32 d128 fwd+bwd"),
}
# per token-head algorithmic work, D = 128, C = 64 (fixed formula; the backward's recompute is not credited)
FLOP_FWD, FLOP_BWD = 181_589, 409_600
BYTES_FWD, BYTES_BWD = 1_032, 1_808


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def synthetic(cfg, device, seed):
    """The configurations' input distributions: q, k, v ~ N(0,1) (bf16); beta = sigmoid(N(0,1));
    g = -exp(U(log 1, log 16)) * softplus(N(0,1)); dO ~ N(0,1) (bf16); s0 ~ N(0, 0.02)."""
    import torch
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    gen = torch.Generator(device=device).manual_seed(seed)
    bf = torch.bfloat16
    t = {}
    t["q"] = torch.randn(B, T, HK, D, generator=gen, device=device).to(bf)
    t["k"] = torch.randn(B, T, HK, D, generator=gen, device=device).to(bf)
    t["v"] = torch.randn(B, T, H, D, generator=gen, device=device).to(bf)
    t["beta"] = torch.sigmoid(torch.randn(B, T, H, generator=gen, device=device))
    t["g"] = (-torch.exp(torch.rand(B, T, H, generator=gen, device=device) * math.log(16.0))
              * torch.nn.functional.softplus(torch.randn(B, T, H, generator=gen, device=device)))
    t["do"] = torch.randn(B, T, H, D, generator=gen, device=device).to(bf)
    t["s0"] = (torch.randn(B, H, D, D, generator=gen, device=device) * 0.02) if cfg["s0"] else None
    t["dsT"] = (torch.randn(B, H, D, D, generator=gen, device=device) * 0.02) if cfg["s0"] else None
    return t


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, power, throttle reasons)."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"gd_clocks_{os.getpid()}.csv")

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_reference(cfg, steps, warmup, sample_batch=1, threads=None):
    """transformers' torch_chunk_gated_delta_rule forward + backward on the CPU over a bounded sample of the workload
    (sample_batch of its B batch rows, all T and H): tokens/s of that sample, median over `steps`."""
    import torch
    from oracle import transformers_ref
    if threads:
        torch.set_num_threads(threads)
    scfg = dict(cfg, B=sample_batch)
    t = synthetic(scfg, "cpu", 1234)
    f = transformers_ref.rule()
    rep = cfg["H"] // cfg["HK"]
    times = []
    for i in range(warmup + steps):
        xs = [t[n].clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")]
        s0 = t["s0"].clone().requires_grad_(True) if t["s0"] is not None else None
        t0 = time.perf_counter()
        qx = xs[0].repeat_interleave(rep, 2) if rep > 1 else xs[0]
        kx = xs[1].repeat_interleave(rep, 2) if rep > 1 else xs[1]
        o, sT = f(qx, kx, xs[2], xs[3], xs[4], chunk_size=64, initial_state=s0, output_final_state=cfg["final"],
                  use_qk_l2norm_in_kernel=True)
        if not cfg["fwd_only"]:
            loss = (o.float() * t["do"].float()).sum()
            if t["dsT"] is not None:
                loss = loss + (sT * t["dsT"]).sum()
            loss.backward()
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    med = statistics.median(times)
    tokens = sample_batch * cfg["T"]
    return {"value": tokens / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"transformers torch_chunk_gated_delta_rule {'fwd' if cfg['fwd_only'] else 'fwd+bwd'} "
                      f"B={sample_batch} of {cfg['B']} (T={cfg['T']}, H={cfg['H']}), median of {steps} "
                      f"after {warmup} warm-up, {med:.3f} s/step",
            "seconds_per_sample": med}


def cpu_config0(steps=5, warmup=1, threads=None):
    """Config 0, the reference's CPU run: transformers' torch_chunk_gated_delta_rule forward only, fp32, B=1, T=256,
    H=4, dk=dv=64, chunk 64, l2-normalised q/k, no initial state, on this host's cores. (The B200 kernels are built for
    head width 128, so this configuration is a CPU-side timing only.)"""
    import torch
    from oracle import transformers_ref
    if threads:
        torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    B, T, H, D = 1, 256, 4, 64
    q, k, v = (torch.randn(B, T, H, D, generator=gen) for _ in range(3))
    beta = torch.sigmoid(torch.randn(B, T, H, generator=gen))
    g = -torch.exp(torch.rand(B, T, H, generator=gen) * math.log(16.0)) * torch.nn.functional.softplus(
        torch.randn(B, T, H, generator=gen))
    f = transformers_ref.rule()
    times = []
    with torch.no_grad():
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            f(q, k, v, g, beta, chunk_size=64, initial_state=None, output_final_state=False,
              use_qk_l2norm_in_kernel=True)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"workload": "c0: B1 T256 H4 d64 fp32 forward (CPU only)", "ms": med * 1e3,
            "tokens_per_s": B * T / med, "cores": torch.get_num_threads(),
            "kind": "reference (transformers torch_chunk_gated_delta_rule)", "steps": steps}


def run_reference(args, cfg):
    """The reference arm: transformers' torch_chunk_gated_delta_rule (the reference torch implementation the drop-in
    replaces) on this host's cores with every thread, on the full configuration (all B batch rows: the same workload
    as the B200 arm), each step one forward + backward; plus config 0's CPU forward as an extra key. Under torchrun
    rank 0 alone runs and prints; the other ranks exit without work."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count()
    res = cpu_reference(cfg, steps=args.steps, warmup=max(1, min(args.warmup, 2)), sample_batch=cfg["B"],
                        threads=threads)
    c0 = cpu_config0(threads=threads)
    line = {"impl": "reference", "metric": METRIC if args.config == 1 else f"gated-delta tokens/s ({cfg['tag']})",
            "value": res["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["seconds_per_sample"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (the configurations' seeded "
            "input distributions)", "config": {"workload": cfg["tag"], "sample": res["sample"],
                                               "same_config": True},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "cpu_config0": c0,
            "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-shard", action="store_true", help="skip the sharded config 3 / config 4 legs")
    ap.add_argument("--profile", action="store_true",
                    help="profiling case for ncu: --steps plain forward+backward calls through the C ABI (no graph, "
                         "no timing, no CPU baseline), then exit; launch order per step: prep, state, prep, state "
                         "(store), bwd_state, bwd_chunk")
    ap.add_argument("--profile-layer", action="store_true",
                    help="profiling case for ncu: --steps rounds of the layer steps' kernels through the C ABI "
                         "(gates, gated norm, convolution path; forward then backward each) at sizes above L2, no "
                         "timing, then exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg)
    if args.profile_layer:
        return profile_layer(args.steps)

    import torch
    import torch.distributed as dist
    from macai_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    lib = _lib.load()
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    t = synthetic(cfg, dev, 1000 + rank)
    flags = _lib.GD_L2NORM | _lib.GD_SCALE_Q
    nbytes = lib.gd_workspace_bytes(B, T, H, HK, D, D, 0 if cfg["fwd_only"] else 1)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    o = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=dev)
    sT = torch.empty(B, H, D, D, dtype=torch.float32, device=dev) if cfg["final"] else None
    dq, dk = torch.empty_like(t["q"]), torch.empty_like(t["k"])
    dv = torch.empty_like(t["v"])
    dg = torch.empty(B, T, H, dtype=torch.float32, device=dev)
    db = torch.empty_like(dg)
    ds0 = torch.empty(B, H, D, D, dtype=torch.float32, device=dev) if cfg["s0"] else None
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    BF = _lib.GD_BFLOAT16
    kernels_per_step = 2 if cfg["fwd_only"] else 6

    def step():
        st = lib.gd_forward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), P(t["s0"]), P(o), P(sT), BF,
                            B, T, H, HK, D, D, flags, P(ws), nbytes, sp)
        _lib.check(st, "gd_forward")
        if not cfg["fwd_only"]:
            st = lib.gd_backward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), P(t["s0"]), P(t["do"]),
                                 P(t["dsT"]), P(dq), P(dk), P(dv), P(dg), P(db), P(ds0), BF, B, T, H, HK, D, D, flags,
                                 P(ws), nbytes, sp)
            _lib.check(st, "gd_backward")

    with torch.cuda.stream(stream):
        for _ in range(args.steps if args.profile else 2):
            step()
    stream.synchronize()
    code = lib.gd_read_error(P(ws), sp, None)
    if code != 0:
        raise RuntimeError(f"device error word {code} after warm-up")
    if args.profile:
        print(json.dumps({"profile": cfg["tag"], "steps": args.steps, "device_status": code}), flush=True)
        return

    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        run = graph.replay
    else:
        def run():
            with torch.cuda.stream(stream):
                step()

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            flush.zero_()
            run()
    stream.synchronize()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with Clocks(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.zero_()
                starts[i].record(stream)
                run()
                ends[i].record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    per_step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = torch.tensor([sum(per_step_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_s = total_ms.item() / 1e3
    tokens_per_step = B * T * world
    value = tokens_per_step * args.steps / total_s

    # ---- the stored-states mode (not the headline): same step with the states kept from the forward
    stored = None
    if not cfg["fwd_only"]:
        stored_ms = stored_mode_ms(lib, t, cfg, flags, ws, nbytes, o, sT, dq, dk, dv, dg, db, ds0, stream, flush,
                                   args.steps, args.warmup)
        if world > 1:
            sm = torch.tensor([stored_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(sm, op=dist.ReduceOp.MAX)
            stored_ms = sm.item()
        stored = {"ms_per_step": stored_ms, "value": tokens_per_step / (stored_ms / 1e3), "unit": "tokens/s",
                  "mode": "RECOMPUTE_STATES=False (the reference's stored mode): the training forward keeps the chunk "
                          "matrices, states and Vn, the backward skips the recompute; same bits as the headline's "
                          "recompute mode"}

    # ---- packed rows (not the headline): the same tokens as N sequences of random lengths in one batch row
    packed = None
    if not cfg["fwd_only"] and rank == 0:
        packed = packed_mode(lib, t, cfg, flags, stream, flush, args.steps, args.warmup)

    # ---- per-kernel timing pass (not the headline): each entry point between events on the stream
    kern = kernel_times(lib, t, cfg, flags, ws, nbytes, o, sT, dq, dk, dv, dg, db, ds0, stream, flush)
    gates = gates_times(lib, dev, stream, flush) if rank == 0 else None
    gnorm = gnorm_times(lib, dev, stream, flush) if rank == 0 else None
    conv = conv_times(lib, dev, stream, flush) if rank == 0 else None
    hbm, tflops, peak_kind = peaks()
    roof = roofline(kern, cfg, hbm, tflops, peak_kind)

    # ---- end to end through the C ABI with host buffers
    e2e = end_to_end(lib, t, cfg, flags, ws, nbytes, stream, args)
    if world > 1:
        e2 = torch.tensor([e2e["seconds"]], dtype=torch.float64, device=dev)
        dist.all_reduce(e2, op=dist.ReduceOp.MAX)
        e2e["seconds"] = e2.item()
    e2e_value = tokens_per_step * e2e["steps"] / e2e["seconds"]
    floor_s = _max_over_ranks(e2e["copy_floor_seconds"], dev, world)

    # ---- the sharded configurations (strong scaling over the ranks; their one-GPU points at N = 1)
    c3 = c4 = None
    if not args.no_shard and args.config == 1:
        c4 = sharded_c4(lib, dev, rank, world, steps=min(args.steps, 5), warmup=3, flush=flush)
        c3 = sharded_c3(lib, dev, rank, world, steps=min(args.steps, 10), warmup=3, flush=flush)

    cpu = cpu0 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference(cfg, steps=3, warmup=1, sample_batch=cfg["B"], threads=os.cpu_count())
        cpu = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        cpu0 = cpu_config0(threads=os.cpu_count())

    step_flops = (FLOP_FWD + (0 if cfg["fwd_only"] else FLOP_BWD)) * B * T * H
    step_bytes = (BYTES_FWD + (0 if cfg["fwd_only"] else BYTES_BWD)) * B * T * H
    step_s = total_s / args.steps
    if rank == 0:
        line = {
            "metric": METRIC if args.config == 1 else f"gated-delta tokens/s ({cfg['tag']})",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_s * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / PUBLISHED_TOKENS_S) if args.config == 1 else None,
            "dtype": "bf16", "data": "synthetic (seeded per rank: q, k, v, dO ~ N(0,1); beta = sigmoid(N(0,1)); "
                                                 "g = -exp(U(0, log 16)) softplus(N(0,1)))",
            "config": {"workload": cfg["tag"], "global_batch": B * world, "seq_len": T, "heads": H,
                       "key_heads": HK, "head_dim": D, "chunk": 64, "parallelism": f"dp{world} over (batch, head)",
                       "l2": "flushed between steps (256 MiB write, outside the per-step events)",
                       "cuda_graph": graph is not None, "per_rank_batch": B,
                       "vs_baseline_ref": "M3 Max Metal fwd+bwd 10.210 ms at B4 T1024 H16 (reference docs)"},
            "step_roofline": {"achieved_tflops": step_flops / step_s / 1e12,
                              "achieved_gbs": step_bytes / step_s / 1e9,
                              "roofline_time_us": max(step_flops / (tflops * 1e12), step_bytes / (hbm * 1e9)) * 1e6,
                              "frac": max(step_flops / (tflops * 1e12), step_bytes / (hbm * 1e9)) / step_s,
                              "peak": f"{peak_kind} MEASURED_PEAKS.json"},
            "roofline": roof,
            "kernels": kern,
            "stored_states": stored,
            "packed": packed,
            "gates": gates,
            "gated_norm": gnorm,
            "conv": conv,
            "cpu_baseline": cpu,
            "cpu_config0": cpu0,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e["seconds"] * 1e3 / e2e["steps"],
                    "copy_floor_ms": floor_s * 1e3 / e2e["steps"],
                    "copy_floor": "the same pipelined host<->device copies with no compute (both directions at once, "
                                  "max over ranks)", "numa_node": e2e["numa"]},
            "c3": c3,
            "c4": c4,
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def slice_inputs(cfg, dev, sl, seed, fwd_only):
    """Inputs of one rank's slice (shard.Slice) of a configuration, each (batch row, key head) unit seeded on its own
    (seed + 1000 b + hk), so that every rank, and a one-GPU run of any subset of rows, builds the same values. A unit
    holds its key head's q, k and the rep value heads it serves (v, g, beta, dO), with the distributions of
    `synthetic`."""
    import torch
    T, H, HK, D = cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    rep = H // HK
    return unit_inputs(T, D, rep, range(sl.b0, sl.b1), range(sl.hk0, sl.hk1), dev, seed, fwd_only)


def unit_inputs(T, D, rep, rows, key_heads, dev, seed, fwd_only):
    """q, k [len(rows), T, len(key_heads), D] bf16, v / dO [.., rep * len(key_heads), D] bf16, g / beta fp32 for the
    listed global batch rows and key heads (the unit seeding of slice_inputs)."""
    import torch
    nb, nk = len(rows), len(key_heads)
    bf = torch.bfloat16
    t = {"q": torch.empty(nb, T, nk, D, dtype=bf, device=dev), "k": torch.empty(nb, T, nk, D, dtype=bf, device=dev),
         "v": torch.empty(nb, T, nk * rep, D, dtype=bf, device=dev),
         "g": torch.empty(nb, T, nk * rep, device=dev), "beta": torch.empty(nb, T, nk * rep, device=dev),
         "do": None if fwd_only else torch.empty(nb, T, nk * rep, D, dtype=bf, device=dev)}
    for i, b in enumerate(rows):
        for j, hk in enumerate(key_heads):
            gen = torch.Generator(device=dev).manual_seed(seed + 1000 * b + hk)
            hs = slice(j * rep, (j + 1) * rep)
            t["q"][i, :, j] = torch.randn(T, D, generator=gen, device=dev).to(bf)
            t["k"][i, :, j] = torch.randn(T, D, generator=gen, device=dev).to(bf)
            t["v"][i, :, hs] = torch.randn(T, rep, D, generator=gen, device=dev).to(bf)
            t["beta"][i, :, hs] = torch.sigmoid(torch.randn(T, rep, generator=gen, device=dev))
            t["g"][i, :, hs] = (-torch.exp(torch.rand(T, rep, generator=gen, device=dev) * math.log(16.0))
                                * torch.nn.functional.softplus(torch.randn(T, rep, generator=gen, device=dev)))
            if not fwd_only:
                t["do"][i, :, hs] = torch.randn(T, rep, D, generator=gen, device=dev).to(bf)
    return t


def _same_bits(a, b):
    """Bitwise equality of two tensors of one dtype and shape (NaNs included)."""
    import torch
    ints = {torch.float32: torch.int32, torch.bfloat16: torch.int16, torch.float16: torch.int16}
    return a.shape == b.shape and a.dtype == b.dtype and bool(torch.equal(a.view(ints[a.dtype]),
                                                                           b.view(ints[b.dtype])))


def _max_over_ranks(x, dev, world):
    import torch
    import torch.distributed as dist
    v = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return v.item()


def sharded_c4(lib, dev, rank, world, steps, warmup, flush):
    """Config 4 (B=64, T=4096, H=32, forward + backward) with its batch rows split over the ranks (strong scaling:
    the job's 262,144 tokens are fixed, each rank computes 64 / N rows through the C ABI, no collective on the data
    path). Timed as the headline: CUDA graph, L2 flushed between steps, barrier + synchronise around the timed region,
    device time maximum over ranks. Then the bit-identity check: every rank's first row of dq, dk, dv, dg, dbeta is
    gathered (NCCL all_gather_into_tensor) and rank 0 computes the same rows (built from the same unit seeds) in one
    call of its own; they must be the same bits."""
    import torch
    import torch.distributed as dist
    from macai_b200 import _lib
    from macai_b200.gated_delta import shard
    cfg = CONFIGS[4]
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    sl = shard.partition(B, H, HK, world, rank)
    assert sl.dim == 0, "config 4 splits batch rows"
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    BF, flags = _lib.GD_BFLOAT16, _lib.GD_L2NORM | _lib.GD_SCALE_Q
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)

    def buffers(t, nb):
        o = torch.empty(nb, T, H, D, dtype=torch.bfloat16, device=dev)
        grads = [torch.empty_like(t["q"]), torch.empty_like(t["k"]), torch.empty_like(t["v"]),
                 torch.empty(nb, T, H, device=dev), torch.empty(nb, T, H, device=dev)]
        nbytes = lib.gd_workspace_bytes(nb, T, H, HK, D, D, 1)
        return o, grads, torch.empty(nbytes, dtype=torch.uint8, device=dev), nbytes

    def step_fn(t, nb, o, grads, ws, nbytes):
        def step():
            _lib.check(lib.gd_forward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), None, P(o), None, BF,
                                      nb, T, H, HK, D, D, flags, P(ws), nbytes, sp), "gd_forward")
            _lib.check(lib.gd_backward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), None, P(t["do"]),
                                       None, *[P(x) for x in grads], None, BF, nb, T, H, HK, D, D, flags, P(ws),
                                       nbytes, sp), "gd_backward")
        return step

    nb = sl.b1 - sl.b0
    t = slice_inputs(cfg, dev, sl, 4000, False)
    o, grads, ws, nbytes = buffers(t, nb)
    step = step_fn(t, nb, o, grads, ws, nbytes)
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            graph.replay()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / steps, dev, world)
    code = lib.gd_read_error(P(ws), sp, None)
    del graph
    # bit identity of the sharded gradients against one call over the same rows
    firsts = [shard.partition(B, H, HK, world, r).b0 for r in range(world)]
    mine = [x[0:1].contiguous() for x in grads]
    gathered = []
    for x in mine:
        buf = torch.empty((world,) + tuple(x.shape[1:]), dtype=x.dtype, device=dev)
        if world > 1:
            dist.all_gather_into_tensor(buf, x)
        else:
            buf.copy_(x)
        gathered.append(buf)
    torch.cuda.synchronize(dev)
    del t, o, grads, ws
    identical = None
    if rank == 0:
        t1 = unit_inputs(T, D, H // HK, firsts, range(HK), dev, 4000, False)
        o1, g1, ws1, nb1 = buffers(t1, world)
        with torch.cuda.stream(stream):
            step_fn(t1, world, o1, g1, ws1, nb1)()
        stream.synchronize()
        identical = all(_same_bits(a, b) for a, b in zip(gathered, g1))
        del t1, o1, g1, ws1
    torch.cuda.empty_cache()
    tokens = B * T
    return {"workload": "c4: B64 T4096 H32 d128 fwd+bwd, batch rows split over the ranks (strong scaling)",
            "rows_per_rank": nb, "ms_per_step": ms, "tokens_per_s": tokens / (ms / 1e3), "steps": steps,
            "l2": "inputs above L2 and flushed between steps", "device_status": code,
            "bit_identical_vs_one_gpu": identical,
            "identity_rows": firsts, "collective": "none on the data path; the identity check gathers one row of "
                                                   "dq/dk/dv/dg/dbeta per rank after timing"}


def sharded_c3(lib, dev, rank, world, steps, warmup, flush):
    """Config 3 (B=1, T=32768, H=32, forward with the final state) with its heads split over the ranks (strong
    scaling: 32 / N heads each), the final states [1, 32, 128, 128] fp32 gathered into every rank by NCCL
    all_gather_into_tensor inside the timed region. Per step (L2 flushed before): the forward through the C ABI,
    then the gather; device time (CUDA events on the launching stream, which the collective joins) maximum over
    ranks, also split into the forward and the gather, so the curve's limit can be named."""
    import torch
    import torch.distributed as dist
    from macai_b200 import _lib
    from macai_b200.gated_delta import shard
    cfg = CONFIGS[3]
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    sl = shard.partition(B, H, HK, world, rank)
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    BF, flags = _lib.GD_BFLOAT16, _lib.GD_L2NORM | _lib.GD_SCALE_Q
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    t = slice_inputs(cfg, dev, sl, 3000, True)
    Hl, HKl = sl.h1 - sl.h0, sl.hk1 - sl.hk0
    o = torch.empty(B, T, Hl, D, dtype=torch.bfloat16, device=dev)
    sT = torch.empty(B, Hl, D, D, device=dev)
    sT_all = torch.empty(world * B * Hl * D * D, device=dev)
    nbytes = lib.gd_workspace_bytes(B, T, Hl, HKl, D, D, 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def fwd():
        _lib.check(lib.gd_forward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), None, P(o), P(sT), BF, B,
                                  T, Hl, HKl, D, D, flags, P(ws), nbytes, sp), "gd_forward")

    def gather():
        if world > 1:
            dist.all_gather_into_tensor(sT_all, sT.reshape(-1))
        else:
            sT_all.copy_(sT.reshape(-1))

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            fwd()
            gather()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for e in evs:
            flush.zero_()
            e[0].record(stream)
            fwd()
            e[1].record(stream)
            gather()
            e[2].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(sum(e[0].elapsed_time(e[2]) for e in evs) / steps, dev, world)
    fwd_ms = _max_over_ranks(sum(e[0].elapsed_time(e[1]) for e in evs) / steps, dev, world)
    gat_ms = _max_over_ranks(sum(e[1].elapsed_time(e[2]) for e in evs) / steps, dev, world)
    code = lib.gd_read_error(P(ws), sp, None)
    # the gathered states hold every rank's heads in rank order: this rank's part is its own
    mine = sT_all.view(world, -1)[rank].view_as(sT)
    gathered_ok = bool(torch.equal(mine, sT))
    del t, o, sT, sT_all, ws
    torch.cuda.empty_cache()
    return {"workload": "c3: B1 T32768 H32 d128 forward + final states, heads split over the ranks (strong scaling)",
            "heads_per_rank": Hl, "ms_per_step": ms, "tokens_per_s": B * T / (ms / 1e3), "forward_ms": fwd_ms,
            "gather_ms": gat_ms, "gather_bytes": world * B * Hl * D * D * 4, "steps": steps,
            "l2": "inputs above L2 and flushed between steps", "device_status": code, "gather_ok": gathered_ok,
            "limit": ("the gather" if gat_ms > fwd_ms else
                      f"the forward's sequential chunk chain ({T // 64} chunks per head in order)")}


def stored_mode_ms(lib, t, cfg, flags, ws, nbytes, o, sT, dq, dk, dv, dg, db, ds0, stream, flush, steps, warmup):
    """Device ms per forward + backward step in the stored-states mode (gd_forward with GD_STORE_STATES, then
    gd_backward with GD_STATES_STORED on the same workspace), CUDA graph, L2 flushed between steps as the headline."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    BF = _lib.GD_BFLOAT16

    def step():
        _lib.check(lib.gd_forward(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), P(t["s0"]), P(o), P(sT),
                                  BF, B, T, H, HK, D, D, flags | _lib.GD_STORE_STATES, P(ws), nbytes, sp), "gd_forward")
        _lib.check(lib.gd_backward(P(t["q"]), P(t["k"]), P(t["v"]), None, P(t["beta"]), None, P(t["do"]), P(t["dsT"]),
                                   P(dq), P(dk), P(dv), P(dg), P(db), P(ds0), BF, B, T, H, HK, D, D,
                                   flags | _lib.GD_STATES_STORED, P(ws), nbytes, sp), "gd_backward")

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            graph.replay()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with torch.cuda.stream(stream):
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            graph.replay()
            ends[i].record(stream)
    stream.synchronize()
    code = lib.gd_read_error(P(ws), sp, None)
    if code != 0:
        raise RuntimeError(f"device error word {code} in the stored-states pass")
    del graph
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / steps


def profile_layer(steps):
    """The layer steps' kernels for an ncu capture: gates over [16, 4096, 32] (bf16 b, a; fp32 A_log, dt_bias),
    the gated norm over 1 M rows of 128 (bf16, frozen weight), the convolution path over [4, 4096, 8192] with the 9B
    widths (bf16, frozen weight); each round runs every forward, then every backward, once. Inputs of 128-512 MB
    each (above the 126 MB L2), about 3 GB in all."""
    import torch
    from macai_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    BF, F32 = _lib.GD_BFLOAT16, _lib.GD_FLOAT32
    gen = torch.Generator(device=dev).manual_seed(3)
    bf = torch.bfloat16
    # gates
    shape, H = (16, 4096, 32), 32
    n = 16 * 4096 * 32
    gb, ga = (torch.randn(shape, generator=gen, device=dev).to(bf) for _ in range(2))
    A_log, dt_bias = torch.rand(H, generator=gen, device=dev) * 2.7, torch.randn(H, generator=gen, device=dev)
    beta, g = torch.empty(shape, device=dev), torch.empty(shape, device=dev)
    dbeta, dg = torch.randn_like(beta), torch.randn_like(g)
    db, da = torch.empty_like(gb), torch.empty_like(ga)
    # gated norm
    rows, D = 1 << 20, 128
    x, z, do = (torch.randn(rows, D, generator=gen, device=dev).to(bf) for _ in range(3))
    w = torch.ones(D, device=dev, dtype=bf)
    o, dx, dz = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
    # convolution path
    B, T, kd, rep = 4, 4096, 2048, 2
    C, hv = 2 * kd + kd * rep, kd // 128 * rep
    cx = torch.randn(B, T, C, generator=gen, device=dev).to(bf)
    cw = (torch.randn(C, 4, generator=gen, device=dev) * 0.3).to(bf)
    cq, ck = (torch.empty(B, T, hv, 128, device=dev, dtype=bf) for _ in range(2))
    cv = torch.empty(B, T, hv, 128, device=dev)
    cdx = torch.empty_like(cx)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(steps):
            _lib.check(lib.gd_gates_fwd(P(gb), P(ga), P(A_log), P(dt_bias), P(beta), P(g), BF, F32, n, H, sp), "gates")
            _lib.check(lib.gd_gnorm_fwd(P(x), P(z), P(w), P(o), BF, BF, rows, D, 1e-6, sp), "gnorm")
            _lib.check(lib.gd_conv_fwd(P(cx), P(cw), P(cq), P(ck), P(cv), BF, BF, B, T, C, kd, 128, rep, 128, sp),
                       "conv")
            _lib.check(lib.gd_gates_bwd(P(gb), P(ga), P(A_log), P(dt_bias), P(dbeta), P(dg), P(db), P(da), None, None,
                                        BF, F32, n, H, None, 0, sp), "gates")
            _lib.check(lib.gd_gnorm_bwd(P(x), P(z), P(w), P(do), P(dx), P(dz), None, BF, BF, rows, D, 1e-6, None, 0,
                                        sp), "gnorm")
            _lib.check(lib.gd_conv_bwd(P(cx), P(cw), P(cq), P(ck), P(cv), P(cdx), None, BF, BF, B, T, C, kd, 128, rep,
                                       128, None, 0, sp), "conv")
    stream.synchronize()
    print(json.dumps({"profile": "layer steps", "steps": steps}), flush=True)


def packed_mode(lib, t, cfg, flags, stream, flush, steps, warmup, nseq=12, seed=5):
    """Forward + backward over packed rows (gd_forward_packed then gd_backward_packed, recompute mode): the config's
    B * T tokens (the same q, k, v, g, beta, dO viewed as one batch row) split into `nseq` sequences of seeded random
    lengths (at least 1 token each, boundaries uniform over the tokens), with per-sequence initial states and state
    gradients; CUDA graph, L2 flushed between steps as the headline. Reports ms per step and tokens/s; every sequence
    starts a new chunk, so the chunk count grows by up to one per sequence over the headline's."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    dev = t["q"].device
    Ttot = B * T
    gen = torch.Generator().manual_seed(seed)
    cuts = torch.randperm(Ttot - 1, generator=gen)[:nseq - 1].sort().values + 1
    cu_host = torch.cat([torch.tensor([0]), cuts, torch.tensor([Ttot])]).to(torch.int32)
    cu = cu_host.to(dev)
    view = lambda x: x.reshape(1, Ttot, *x.shape[2:])
    q, k, v, g, beta, do = (view(t[n]) for n in ("q", "k", "v", "g", "beta", "do"))
    s0 = torch.randn(nseq, H, D, D, device=dev) * 0.02
    dsT = torch.randn(nseq, H, D, D, device=dev) * 0.02
    o = torch.empty_like(v)
    sT = torch.empty_like(s0)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg, db = torch.empty_like(g), torch.empty_like(beta)
    ds0 = torch.empty_like(s0)
    nb = lib.gd_workspace_bytes_packed(nseq, Ttot, H, HK, D, D, 1)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    BF = _lib.GD_BFLOAT16

    def step():
        _lib.check(lib.gd_forward_packed(P(q), P(k), P(v), P(g), P(beta), P(s0), P(o), P(sT), P(cu), nseq, BF, Ttot, H,
                                         HK, D, D, flags, P(ws), nb, sp), "gd_forward_packed")
        _lib.check(lib.gd_backward_packed(P(q), P(k), P(v), P(g), P(beta), P(s0), P(do), P(dsT), P(dq), P(dk), P(dv),
                                          P(dg), P(db), P(ds0), P(cu), nseq, BF, Ttot, H, HK, D, D, flags, P(ws), nb,
                                          sp), "gd_backward_packed")

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            flush.zero_()
            graph.replay()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with torch.cuda.stream(stream):
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            graph.replay()
            ends[i].record(stream)
    stream.synchronize()
    code = lib.gd_read_error(P(ws), sp, None)
    if code != 0:
        raise RuntimeError(f"device error word {code} in the packed-rows pass")
    del graph
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / steps
    lengths = (cu_host[1:] - cu_host[:-1]).tolist()
    return {"ms_per_step": ms, "value": Ttot / (ms / 1e3), "unit": "tokens/s", "sequences": nseq,
            "lengths": lengths, "chunks": int(sum((n + 63) // 64 for n in lengths)),
            "mode": "cu_seqlens: the config's tokens as one batch row of sequences with random boundaries (seeded), "
                    "per-sequence states; fwd + bwd, recompute mode"}


def gates_times(lib, dev, stream, flush, iters=10):
    """The layer's gates (gd_gates_fwd / gd_gates_bwd, bf16 b and a, fp32 A_log and dt_bias, frozen gate weights as in
    LoRA training: no per-head sums) at config 1's [B, T, H] and at config 4's [64, 4096, 32]: device microseconds per
    call (CUDA events, L2 flushed before each) and HBM bandwidth from the algorithmic bytes (forward: b, a read, beta, g
    written = 12 B per element; backward: b, a, dbeta, dg read, db, da written = 16 B per element)."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    hbm, _, _ = peaks()
    out = {}
    for tag, shape in (("c1", (4, 1024, 16)), ("c4", (64, 4096, 32))):
        n, H = shape[0] * shape[1] * shape[2], shape[2]
        gen = torch.Generator(device=dev).manual_seed(7)
        b = torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)
        a = torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)
        A_log = torch.rand(H, generator=gen, device=dev) * 2.7
        dt_bias = torch.randn(H, generator=gen, device=dev)
        beta = torch.empty(shape, device=dev)
        g = torch.empty(shape, device=dev)
        dbeta, dg = torch.randn_like(beta), torch.randn_like(g)
        db, da = torch.empty_like(b), torch.empty_like(a)
        BF, F32 = _lib.GD_BFLOAT16, _lib.GD_FLOAT32

        def fwd():
            _lib.check(lib.gd_gates_fwd(P(b), P(a), P(A_log), P(dt_bias), P(beta), P(g), BF, F32, n, H, sp), "gates")

        def bwd():
            _lib.check(lib.gd_gates_bwd(P(b), P(a), P(A_log), P(dt_bias), P(dbeta), P(dg), P(db), P(da), None, None,
                                        BF, F32, n, H, None, 0, sp), "gates")
        res = {"elements": n}
        for name, f, per in (("fwd", fwd, 12), ("bwd", bwd, 16)):
            with torch.cuda.stream(stream):
                f()
                tot = 0.0
                for _ in range(iters):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    f()
                    e1.record(stream)
                    e1.synchronize()
                    tot += e0.elapsed_time(e1)
            us = tot / iters * 1e3
            gbs = per * n / (us * 1e-6) / 1e9
            res[name] = {"us": us, "gbs": gbs, "frac_hbm": gbs / hbm}
        out[tag] = res
    return out


def gnorm_times(lib, dev, stream, flush, iters=10):
    """The gated RMSNorm on the rule's output (gd_gnorm_fwd / gd_gnorm_bwd, bf16 x and z, bf16 weight frozen as in
    LoRA training: no weight gradient) over config 1's and config 4's [B * T * H, 128] rows: device microseconds per
    call (CUDA events, L2 flushed before each) and HBM bandwidth from the algorithmic bytes (forward: x, z read, o
    written = 6 B per element; backward: x, z, dout read, dx, dz written = 10 B per element)."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    hbm, _, _ = peaks()
    BF = _lib.GD_BFLOAT16
    out = {}
    for tag, rows in (("c1", 4 * 1024 * 16), ("c4", 64 * 4096 * 32)):
        D = 128
        gen = torch.Generator(device=dev).manual_seed(9)
        x = torch.randn(rows, D, generator=gen, device=dev, dtype=torch.bfloat16)
        z = torch.randn(rows, D, generator=gen, device=dev, dtype=torch.bfloat16)
        do = torch.randn(rows, D, generator=gen, device=dev, dtype=torch.bfloat16)
        w = (torch.randn(D, generator=gen, device=dev) * 0.1 + 1).to(torch.bfloat16)
        o, dx, dz = torch.empty_like(x), torch.empty_like(x), torch.empty_like(z)

        def fwd():
            _lib.check(lib.gd_gnorm_fwd(P(x), P(z), P(w), P(o), BF, BF, rows, D, 1e-6, sp), "gnorm")

        def bwd():
            _lib.check(lib.gd_gnorm_bwd(P(x), P(z), P(w), P(do), P(dx), P(dz), None, BF, BF, rows, D, 1e-6, None, 0,
                                        sp), "gnorm")
        res = {"rows": rows, "width": D}
        for name, f, per in (("fwd", fwd, 6), ("bwd", bwd, 10)):
            with torch.cuda.stream(stream):
                f()
                tot = 0.0
                for _ in range(iters):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    f()
                    e1.record(stream)
                    e1.synchronize()
                    tot += e0.elapsed_time(e1)
            us = tot / iters * 1e3
            gbs = per * rows * D / (us * 1e-6) / 1e9
            res[name] = {"us": us, "gbs": gbs, "frac_hbm": gbs / hbm}
        out[tag] = res
        del x, z, do, o, dx, dz
    return out


def conv_times(lib, dev, stream, flush, iters=5):
    """The convolution path (gd_conv_fwd / gd_conv_bwd, bf16 x and weight, the weight frozen as in LoRA training) at
    config 1's tokens with Qwen3.5-0.8B's widths (C = 6144: 16 key heads and 16 value heads of 128) and at config 4's
    tokens with 9B's (C = 8192: 16 key heads serving 32 value heads): device microseconds per call (CUDA events, L2
    flushed before each) and HBM bandwidth from the algorithmic bytes (forward: x read, q and k written in bf16 with
    the key heads repeated, v written in fp32; backward: x, dq, dk, dv read, dx written)."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    hbm, _, _ = peaks()
    BF = _lib.GD_BFLOAT16
    out = {}
    for tag, (B, T, kd, rep) in (("c1", (4, 1024, 2048, 1)), ("c4", (64, 4096, 2048, 2))):
        dk = dv = 128
        vd = kd * rep
        C = 2 * kd + vd
        hv = kd // dk * rep
        gen = torch.Generator(device=dev).manual_seed(11)
        x = torch.randn(B, T, C, generator=gen, device=dev, dtype=torch.bfloat16)
        w = (torch.randn(C, 4, generator=gen, device=dev) * 0.3).to(torch.bfloat16)
        q = torch.empty(B, T, hv, dk, device=dev, dtype=torch.bfloat16)
        k = torch.empty_like(q)
        v = torch.empty(B, T, hv, dv, device=dev)
        dx = torch.empty_like(x)

        def fwd():
            _lib.check(lib.gd_conv_fwd(P(x), P(w), P(q), P(k), P(v), BF, BF, B, T, C, kd, dk, rep, dv, sp), "conv")

        def bwd():  # the forward's outputs stand in for the cotangents (same shapes and dtypes)
            _lib.check(lib.gd_conv_bwd(P(x), P(w), P(q), P(k), P(v), P(dx), None, BF, BF, B, T, C, kd, dk, rep, dv,
                                       None, 0, sp), "conv")
        tokens = B * T
        per_fwd = tokens * (2 * C + 2 * 2 * hv * dk + 4 * hv * dv)
        per_bwd = tokens * (2 * C + 2 * 2 * hv * dk + 4 * hv * dv + 2 * C)
        res = {"tokens": tokens, "channels": C, "rep": rep}
        for name, f, nbytes in (("fwd", fwd, per_fwd), ("bwd", bwd, per_bwd)):
            with torch.cuda.stream(stream):
                f()
                tot = 0.0
                for _ in range(iters):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    f()
                    e1.record(stream)
                    e1.synchronize()
                    tot += e0.elapsed_time(e1)
            us = tot / iters * 1e3
            gbs = nbytes / (us * 1e-6) / 1e9
            res[name] = {"us": us, "gbs": gbs, "frac_hbm": gbs / hbm}
        out[tag] = res
        del x, q, k, v, dx
    return out


def kernel_times(lib, t, cfg, flags, ws, nbytes, o, sT, dq, dk, dv, dg, db, ds0, stream, flush, iters=5):
    """Average device time of each kernel (entry point) of one step, CUDA events on the launching stream, L2 flushed
    before each step's sequence."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    BF = _lib.GD_BFLOAT16
    # the forward pair in the forward-only layout, as gd_forward runs it (the layout follows the size passed)
    nf = lib.gd_workspace_bytes(B, T, H, HK, D, D, 0)
    seq = [("prep", lambda: lib.gd_prep(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), BF, B, T, H, HK, D, D,
                                        flags, P(ws), nf, sp)),
           ("fwd_state", lambda: lib.gd_fwd_state(P(t["s0"]), P(o), P(sT), BF, B, T, H, HK, D, D, flags, P(ws), nf,
                                                  sp))]
    if not cfg["fwd_only"]:
        seq += [("prep(bwd)", lambda: lib.gd_prep(P(t["q"]), P(t["k"]), P(t["v"]), P(t["g"]), P(t["beta"]), BF, B, T,
                                                  H, HK, D, D, flags, P(ws), nbytes, sp)),
                ("fwd_state(store)", lambda: lib.gd_fwd_state(P(t["s0"]), None, None, BF, B, T, H, HK, D, D,
                                                              flags | _lib.GD_STORE_STATES, P(ws), nbytes, sp)),
                ("bwd_state", lambda: lib.gd_bwd_state(P(t["do"]), P(t["dsT"]), P(ds0), BF, B, T, H, HK, D, D, flags,
                                                       P(ws), nbytes, sp)),
                ("bwd_chunk", lambda: lib.gd_bwd_chunk(P(t["q"]), P(t["k"]), P(t["v"]), P(t["beta"]), P(t["do"]),
                                                       P(dq), P(dk), P(dv), P(dg), P(db), BF, B, T, H, HK, D, D, flags,
                                                       P(ws), nbytes, sp))]
    acc = {name: 0.0 for name, _ in seq}
    with torch.cuda.stream(stream):
        for it in range(iters + 1):
            flush.zero_()
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(seq) + 1)]
            evs[0].record(stream)
            for i, (name, f) in enumerate(seq):
                _lib.check(f(), name)
                evs[i + 1].record(stream)
            stream.synchronize()
            if it > 0:
                for i, (name, _) in enumerate(seq):
                    acc[name] += evs[i].elapsed_time(evs[i + 1])
    return {name: acc[name] / iters * 1e3 for name in acc}  # microseconds


def roofline(kern, cfg, hbm, tflops, peak_kind):
    """The dominant kernel against its bound. Algorithmic work per launch (per token-head unit, D = 128, C = 64),
    derived from the same dense counts as the step's FLOP formula:
      fwd_state        6 D^2 + 2 C D   = 114,688 FLOP   (W S, Q S, K^T Vn; M Vn)     bytes: q, k bf16 + o bf16
      bwd_state        6 D^2 + 2 C D   = 114,688 FLOP   (K dS, Q^T dO, W^T dVn; M^T dO)
      bwd_chunk        10 D^2 + 16 C D + 4 C^2 = 311,296 FLOP
      prep             8 C D           =  65,536 FLOP   (Q K^T, K K^T, W, U: four C x C x D products)
    and HBM bytes per token-head of the kernel's algorithmic inputs and outputs (bf16 q/k/v/do/o/grads 256 B each row
    of 128, fp32 g/beta/dg/dbeta 4 B)."""
    D, C = cfg["D"], 64
    per = {
        "prep": (4 * C * D * 2, 3 * 2 * D + 8),
        "prep(bwd)": (4 * C * D * 2, 3 * 2 * D + 8),
        "fwd_state": (6 * D * D + 2 * C * D, 2 * 2 * D + 2 * D),
        "fwd_state(store)": (6 * D * D + 2 * C * D, 2 * 2 * D),
        "bwd_state": (6 * D * D + 2 * C * D, 2 * 2 * D + 2 * D),
        "bwd_chunk": (10 * D * D + 16 * C * D + 4 * C * C, 2 * D * 7 + 16),
    }
    name = max(kern, key=kern.get)
    units = cfg["B"] * cfg["T"] * cfg["H"]
    flop, byts = per[name]
    dur = kern[name] * 1e-6
    a_t = flop * units / dur / 1e12
    a_b = byts * units / dur / 1e9
    traffic = measured_traffic(name, cfg)
    extra = {"traffic_unit": "DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, cold cache)",
             "traffic_source": TRAFFIC_FILE if traffic is not None else None,
             "algorithmic_bytes": byts * units, "algorithmic_flop": flop * units}
    if a_t / tflops >= a_b / hbm:
        return {"kernel": name, "bound": "tensor", "achieved": a_t, "peak": tflops, "unit": "TFLOP/s",
                "frac": a_t / tflops, "traffic": traffic, "peak_source": peak_kind, "duration_us": kern[name],
                "hbm_frac": a_b / hbm, **extra}
    return {"kernel": name, "bound": "hbm", "achieved": a_b, "peak": hbm, "unit": "GB/s", "frac": a_b / hbm,
            "traffic": traffic, "peak_source": peak_kind, "duration_us": kern[name], "tensor_frac": a_t / tflops,
            **extra}


TRAFFIC_FILE = "profiles/bwd_chunk_c1_dram.json"


def measured_traffic(kernel, cfg):
    """DRAM bytes per launch of the dominant kernel from the committed ncu capture summary, when it covers this
    kernel and workload (the capture cannot run inside the timed bench); None otherwise."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), TRAFFIC_FILE)
    try:
        with open(path) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None
    if rec.get("kernel") != kernel or not rec.get("workload", "").startswith(cfg["tag"].split(":")[0] + ":"):
        return None
    return rec["dram_bytes_read"] + rec["dram_bytes_write"]


def bind_to_gpu_numa(index):
    """On a host with more than one NUMA node, restrict this process to the CPUs of the node its GPU hangs off (so its
    pinned host buffers, touched after this, land in that node's memory). Returns the node, or None when the host has
    one node or the topology cannot be read (then nothing changes)."""
    import glob
    nodes = glob.glob("/sys/devices/system/node/node[0-9]*")
    if len(nodes) < 2:
        return None
    try:
        out = subprocess.run(["nvidia-smi", f"--id={index}", "--query-gpu=pci.bus_id", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=20).stdout.strip().lower()
        bus = out[-12:] if len(out) >= 12 else out  # "0000:xx:yy.z"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
        os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


def end_to_end(lib, t, cfg, flags, ws, nbytes, stream, args):
    """The step through the C ABI for a caller holding host buffers: every step copies its inputs from pinned host
    memory to the device, runs forward + backward, and copies every output back to pinned host memory, all inside the
    timed region. As an input pipeline would, the steps overlap: step i's inputs go in on one copy stream while step
    i - 1 computes and step i - 2's outputs come back on another (two buffer sets, ordered by events; host-to-device
    and device-to-host copies use separate engines). A step's inputs live in one pinned host buffer and one device
    buffer (a view per tensor, 256-byte aligned), and so do its outputs: one copy each way per step (one 68 MB copy
    runs at ~55 GB/s where the same bytes as six tensors took twice as long)."""
    import torch
    from macai_b200 import _lib
    P = lambda x: None if x is None else ctypes.c_void_p(x.data_ptr())
    sp = ctypes.c_void_p(stream.cuda_stream)
    dev = t["q"].device
    B, T, H, HK, D = cfg["B"], cfg["T"], cfg["H"], cfg["HK"], cfg["D"]
    names_in = [n for n in ("q", "k", "v", "g", "beta", "s0", "do", "dsT") if t[n] is not None]
    if cfg["fwd_only"]:
        names_in = [n for n in names_in if n not in ("do", "dsT")]
    specs_in = [(n, t[n].shape, t[n].dtype) for n in names_in]
    f32, bf = torch.float32, torch.bfloat16
    specs_out = [("o", (B, T, H, D), bf)] + ([("sT", (B, H, D, D), f32)] if cfg["final"] else [])
    if not cfg["fwd_only"]:
        specs_out += [("dq", tuple(t["q"].shape), bf), ("dk", tuple(t["k"].shape), bf), ("dv", tuple(t["v"].shape), bf),
                      ("dg", tuple(t["g"].shape), f32), ("db", tuple(t["g"].shape), f32)]
        specs_out += [("ds0", (B, H, D, D), f32)] if cfg["s0"] else []

    def packed_set(specs, **kw):
        """One uint8 buffer and a view per tensor (256-byte aligned offsets)."""
        offs, at = [], 0
        for _, shape, dt in specs:
            offs.append(at)
            n = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            at += (n + 255) // 256 * 256
        buf = torch.empty(at, dtype=torch.uint8, **kw)
        views = {}
        for (name, shape, dt), off in zip(specs, offs):
            n = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            views[name] = buf[off:off + n].view(dt).view(shape)
        return buf, views

    numa = bind_to_gpu_numa(dev.index)  # before the pinned buffers are touched: their pages land on that node
    host_in_buf, host_in = packed_set(specs_in, pin_memory=True)
    for n in names_in:
        host_in[n].copy_(t[n].cpu())
    dev_in = [packed_set(specs_in, device=dev) for _ in range(2)]
    outs = [packed_set(specs_out, device=dev) for _ in range(2)]
    host_out = [packed_set(specs_out, pin_memory=True) for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in host_in.values())
    d2h = sum(x.numel() * x.element_size() for x in host_out[0][1].values())
    BF = _lib.GD_BFLOAT16
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = lambda: torch.cuda.Event()
    in_ready, comp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    used = [False, False]

    def one(i):
        b = i & 1
        dbuf, d = dev_in[b]
        obuf, o = outs[b]
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(comp_done[b])  # step i - 2 has finished reading these inputs
            dbuf.copy_(host_in_buf, non_blocking=True)
            in_ready[b].record(s_in)
        stream.wait_event(in_ready[b])
        if used[b]:
            stream.wait_event(out_done[b])  # step i - 2's outputs have been copied out
        st = lib.gd_forward(P(d["q"]), P(d["k"]), P(d["v"]), P(d["g"]), P(d["beta"]), P(d.get("s0")), P(o["o"]),
                            P(o.get("sT")), BF, B, T, H, HK, D, D, flags, P(ws), nbytes, sp)
        _lib.check(st, "gd_forward")
        if not cfg["fwd_only"]:
            st = lib.gd_backward(P(d["q"]), P(d["k"]), P(d["v"]), P(d["g"]), P(d["beta"]), P(d.get("s0")),
                                 P(d["do"]), P(d.get("dsT")), P(o["dq"]), P(o["dk"]), P(o["dv"]), P(o["dg"]),
                                 P(o["db"]), P(o.get("ds0")), BF, B, T, H, HK, D, D, flags, P(ws), nbytes, sp)
            _lib.check(st, "gd_backward")
        comp_done[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[b])
            host_out[b][0].copy_(obuf, non_blocking=True)
            out_done[b].record(s_out)
        used[b] = True

    # 30 steps whatever --steps says (~50 ms): the pipeline's fill (the first inputs in) and drain (the last outputs
    # out) are inside the timed region once, so a longer run reports the pipeline's rate more closely
    steps = 30
    for i in range(2):
        one(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(steps):
        one(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(stream)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    # the copy floor of the same run: the same pipelined copies (each step's inputs in on s_in, outputs out on s_out,
    # both directions at once, two buffer sets) with no compute between them
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s_in)
    s_out.wait_stream(s_in)
    for i in range(steps):
        b = i & 1
        with torch.cuda.stream(s_in):
            dev_in[b][0].copy_(host_in_buf, non_blocking=True)
        with torch.cuda.stream(s_out):
            host_out[b][0].copy_(outs[b][0], non_blocking=True)
    s_out.wait_stream(s_in)
    f1.record(s_out)
    torch.cuda.synchronize(dev)
    return {"seconds": e0.elapsed_time(e1) / 1e3, "steps": steps, "h2d": h2d, "d2h": d2h,
            "copy_floor_seconds": f0.elapsed_time(f1) / 1e3, "numa": numa}


if __name__ == "__main__":
    main()
