#!/usr/bin/env python
"""Benchmark: FP8 128x128 block-scaled MoE layer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--M 64] [--hot 0]

Prints ONE JSON line (rank 0). A step is one MoE layer forward over the
synthetic GLM-5-like decode batch (M=64 tokens by default: H=6144, I=2048,
E=256 experts, top-8 sigmoid router, FP8 e4m3 weights with fp32 128x128 block
scales, 1x128 activation scales, bf16 in/out).

  value       tokens/s over all ranks, inputs resident in HBM, the launches of
              the layer (route, gather+quant, both grouped-GEMM stages in one
              launch, top-k reduce) timed with CUDA events on their stream;
  e2e         the same metric through the public API moe_decode_megakernel_full
              with host (pinned) inputs copied in (one copy of the packed
              hidden rows, ids and weights) and the output copied out inside
              the timed region, every step; the copies run on their own
              stream with two buffer sets, overlapping the neighbouring
              steps' layers as a serving loop would;
  roofline    the dominant kernel (the grouped GEMMs) against measured HBM
              bandwidth;
  cpu_baseline the fp32 CPU oracle on a bounded sample of experts (rank 0, N=1),
              with the GPU layer run on the same sample as a parity check;
  sweep       (N=1) the other single-GPU workloads of the benchmark set on the
              same weights: decode M = 128..1024, M = 1024 with 16 hot experts,
              prefill M = 2048/4096/8192, each with its roofline fraction.
--impl reference times that CPU path alone (the reference is a Python/Triton
package for AMD GPUs; its algorithm is restated by the oracle).

N > 1 (torchrun, one rank per GPU) runs the expert-parallel layer: E/N experts
and M tokens per GPU (weak scaling), exchanged by the kernels through peer
memory (or NCCL all-to-alls with --exchange nccl). The line carries a parity
record (every rank's output against the single-GPU layer over all experts, and
the other exchange form bit for bit) and a config5 record: 8,192 tokens in
total split over the ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE layer tokens/s + HBM GB/s at M=64–1024, FP8 128x128 blockscale, B200"
# Dense FP8 GEMM throughput measured on this pool (torch._scaled_mm, 8192^3,
# e4m3 in, bf16 out, best of 10): the tensor roofline of token-major tiles.
FP8_PEAK_TFLOPS = 3139.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--M", type=int, default=64, help="tokens per GPU")
    ap.add_argument("--hot", type=int, default=0, help="experts with +2.0 router bias (skewed load)")
    ap.add_argument("--experts", type=int, default=256, help="routed experts (fewer only for small profiles)")
    ap.add_argument("--tile", type=int, default=0, help="tokens per GEMM unit (0 = the library's choice)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample-experts", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="N > 1: tokens exchanged by the kernels through peer memory, or by NCCL all-to-alls")
    ap.add_argument("--split", action="store_true", help="the two GEMM stages as two launches (default: one)")
    ap.add_argument("--layer-launch", action="store_true",
                    help="small batches: gather, experts and reduce in one launch (default: three)")
    ap.add_argument("--sweep-steps", type=int, default=10, help="timed steps per sweep / config5 workload")
    ap.add_argument("--no-sweep", action="store_true", help="N=1: skip the sweep record")
    ap.add_argument("--no-config5", action="store_true", help="N>1: skip the config5 record")
    ap.add_argument("--no-parity", action="store_true", help="N>1: skip the parity record")
    ap.add_argument("--no-eplb", action="store_true", help="N>1: skip the hot-expert replication record")
    return ap.parse_args(argv)


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(name: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/<name>.txt),
    line 'dram_bytes_per_launch: N'."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1]))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples of one GPU, kept for the timed region."""

    FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]
    REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.samples = []  # (time, sm_mhz, max_mhz, reasons)
        self.windows = []

    def _reader(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                sm, smax = float(parts[0]), float(parts[1])
            except ValueError:
                continue
            act = {n for n, v in zip(self.REASONS, parts[3:]) if v.lower().startswith("active")}
            self.samples.append((time.monotonic(), sm, smax, act))

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        threading.Thread(target=self._reader, daemon=True).start()
        t0 = time.monotonic()
        while not self.samples and time.monotonic() - t0 < 5.0:
            time.sleep(0.02)

    def mark(self):
        return time.monotonic()

    def window(self, t0, t1, group="main"):
        self.windows.append((t0, t1, group))

    def stop(self):
        """Stops sampling; returns the summary of the "main" windows."""
        if self.proc is None:
            return None
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        return self.summary("main")

    def summary(self, group):
        wins = [(a, b) for a, b, g in self.windows if g == group]
        sel = [s for s in self.samples if any(a - 0.06 <= s[0] <= b + 0.06 for a, b in wins)]
        if not sel and self.samples and wins:
            mid = wins[0][0]
            sel = [min(self.samples, key=lambda s: abs(s[0] - mid))]
        if not sel:
            return None
        reasons = sorted(set().union(*[s[3] for s in sel]))
        return {"sm_mhz": statistics.median(s[1] for s in sel), "sm_max_mhz": max(s[2] for s in sel),
                "reasons": reasons, "samples": len(sel)}


def dist_setup(backend):
    import torch.distributed as dist
    from datetime import timedelta

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            import torch

            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
            torch.cuda.set_device(kw["device_id"])
        dist.init_process_group(backend, timeout=timedelta(seconds=120), **kw)
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, local, ws


def layer_bytes(shape, active, pairs):
    """Algorithmic HBM bytes of one layer step: every active expert's fp8
    weights and block scales once, bf16 hidden in and bf16 out."""
    from trials_b200 import synth

    w = active * (synth.weight_bytes_per_expert(shape.H, shape.I) + synth.scale_bytes_per_expert(shape.H, shape.I))
    return w + shape.M * shape.H * 2 * 2


def packed_inputs(*tensors):
    """One pinned host buffer and one device buffer holding the step's input
    tensors back to back (16-byte aligned), so that each step copies its inputs
    in with a single host-to-device copy. -> (host, device, device views)."""
    import torch

    offs, off = [], 0
    for t in tensors:
        offs.append(off)
        off += (t.numel() * t.element_size() + 15) // 16 * 16
    host = torch.empty(off, dtype=torch.uint8).pin_memory()
    dev = torch.empty(off, dtype=torch.uint8, device=tensors[0].device)
    views = []
    for t, o in zip(tensors, offs):
        n = t.numel() * t.element_size()
        host[o:o + n].copy_(t.contiguous().view(-1).view(torch.uint8).cpu())
        views.append(dev[o:o + n].view(t.dtype).view(t.shape))
    return host, dev, views


def pipelined_e2e(inputs, layer, out_shape, steps, warmup, sync):
    """End-to-end steps through the public API with host buffers. Every step
    copies its inputs in from pinned host memory (one copy of the packed
    tensors) and its (M, H) bf16 result back to pinned host memory. The input
    and result copies run on two streams of their own with two buffer sets, so
    that step k+1's input copy and step k-1's result copy overlap step k's
    layer (as a serving loop overlaps them); the timed region starts before
    the first input copy and ends after the last result copy. layer(views) runs one layer on the device
    input views and returns its output. sync() is called on both sides of the
    timed region (barrier + synchronise). -> (ms per step, h2d bytes, d2h
    bytes)."""
    import torch

    comp = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    slots = []
    for _ in range(2):
        host, dev, views = packed_inputs(*inputs)
        slots.append({"host": host, "dev": dev, "views": views, "out": None,
                      "out_host": torch.empty(out_shape, dtype=torch.bfloat16).pin_memory(),
                      "in_ready": torch.cuda.Event(), "computed": torch.cuda.Event(), "out_done": torch.cuda.Event(),
                      "used": False})

    def step(k):
        sl = slots[k % 2]
        with torch.cuda.stream(h2d):
            if sl["used"]:
                h2d.wait_event(sl["computed"])  # the layer two steps back has read these inputs
            sl["dev"].copy_(sl["host"], non_blocking=True)
            sl["in_ready"].record(h2d)
        comp.wait_event(sl["in_ready"])
        if sl["used"]:
            comp.wait_event(sl["out_done"])  # the result two steps back is on the host: its buffer may go
        sl["out"] = layer(sl["views"])
        sl["computed"].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(sl["computed"])
            sl["out_host"].copy_(sl["out"], non_blocking=True)
            sl["out_done"].record(d2h)
        sl["used"] = True

    for k in range(warmup):
        step(k)
    comp.wait_stream(h2d)
    comp.wait_stream(d2h)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sync()
    start.record(comp)
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    for k in range(steps):
        step(warmup + k)
    comp.wait_stream(h2d)
    comp.wait_stream(d2h)
    end.record(comp)
    sync()
    return start.elapsed_time(end) / steps, slots[0]["host"].numel(), slots[0]["out_host"].numel() * 2


def gemm2_bytes(shape, active, pairs):
    """Algorithmic bytes of one GEMM2 launch: w2 + its scales of every active
    expert, the fp8 inter rows and scales read, the bf16 weighted rows written."""
    H, I = shape.H, shape.I
    w = active * (H * I + 4 * (H // 128) * (I // 128))
    return w + pairs * (I + 4 * I // 128) + pairs * H * 2


def layer_inputs(shape, M, hot, seed, device):
    """Seeded router (logits N(0,1), +hot_bias on the first `hot` experts, then
    the shape's scoring, top-k, renormalised) and bf16 hidden rows N(0,1) of M
    tokens -> (hidden, topk_weights, topk_ids) on `device`."""
    import torch

    from trials_b200 import synth

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    logits = torch.randn(M, shape.E, generator=g, device=device)
    if hot:
        logits[:, :hot] += shape.hot_bias
    tw, ids = synth.make_router(logits, shape.topk, shape.scoring)
    hidden = torch.randn(M, shape.H, generator=g, device=device).to(torch.bfloat16)
    return hidden, tw, ids


def rel_l2(a, b) -> float:
    """||a - b|| / ||b|| in fp32 (on the tensors' device)."""
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def experts_roofline(shape, active, pairs, ms, hbm_peak):
    """Roofline of the experts launch(es) (both grouped-GEMM stages): HBM side
    (algorithmic bytes of both stages, against the measured copy peak) and
    tensor side (2*pairs*3*I*H flops, against the measured FP8 GEMM peak);
    `attainable` = the slower of the two floors over the measured time."""
    nbytes = gemm1_bytes(shape, active, pairs) + gemm2_bytes(shape, active, pairs)
    flops = 2.0 * pairs * 3 * shape.I * shape.H
    t = ms / 1e3
    t_hbm, t_tc = nbytes / (hbm_peak * 1e9), flops / (FP8_PEAK_TFLOPS * 1e12)
    return {"bound": "hbm" if t_hbm >= t_tc else "tensor", "experts_ms": ms,
            "hbm_gbs": nbytes / t / 1e9, "hbm_frac": nbytes / t / 1e9 / hbm_peak,
            "tflops": flops / t / 1e12, "tensor_frac": flops / t / 1e12 / FP8_PEAK_TFLOPS,
            "attainable_frac": max(t_hbm, t_tc) / t, "algorithmic_bytes": nbytes, "algorithmic_flops": flops}


def gemm1_bytes(shape, active, pairs):
    """Algorithmic bytes of one GEMM1 launch: w13 + its scales of every active
    expert, the routed fp8 activation rows and scales read, the fp8 inter rows
    and scales written."""
    H, I = shape.H, shape.I
    w = active * (2 * I * H + 4 * (2 * I // 128) * (H // 128))
    return w + pairs * (H + 4 * H // 128) + pairs * (I + 4 * I // 128)


# ----------------------------------------------------------------------------
# CPU path (oracle): baseline and reference arm
# ----------------------------------------------------------------------------
def cpu_sample_setup(shape, n_sample, seed):
    """A bounded CPU sample of the workload: the router over all M tokens, and
    weights for only the first n_sample active experts."""
    import torch

    from oracle import moe_oracle as orc
    from trials_b200 import synth

    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(shape.M, shape.E, generator=g)
    if shape.hot_experts:
        logits[:, : shape.hot_experts] += shape.hot_bias
    tw, ids = synth.make_router(logits, shape.topk, shape.scoring)
    active = torch.unique(ids).tolist()
    sample = active[:n_sample]
    emap = torch.full((shape.E,), -1, dtype=torch.int32)
    emap[torch.tensor(sample)] = torch.arange(len(sample), dtype=torch.int32)
    w13 = (torch.randn(len(sample), 2 * shape.I, shape.H, generator=g) * 0.02).to(torch.bfloat16)
    w13_q, w13_s = orc.per_block_quant_fp8(w13)
    del w13
    w2 = (torch.randn(len(sample), shape.H, shape.I, generator=g) * 0.02).to(torch.bfloat16)
    w2_q, w2_s = orc.per_block_quant_fp8(w2)
    del w2
    hidden = torch.randn(shape.M, shape.H, generator=g).to(torch.bfloat16)
    return dict(hidden=hidden, tw=tw, ids=ids, emap=emap, n=len(sample), active=len(active), w13_q=w13_q,
                w13_s=w13_s, w2_q=w2_q, w2_s=w2_s)


def cpu_sample_run(s):
    """One timed pass of the fp32 oracle over the sampled experts; returns
    (seconds for the sample, the oracle's output)."""
    import torch

    from oracle import moe_oracle as orc

    t0 = time.perf_counter()
    out = orc.moe_layer(s["hidden"], s["w13_q"], s["w13_s"], s["w2_q"], s["w2_s"], s["tw"], s["ids"],
                        expert_map=s["emap"].numpy(), num_local=s["n"], dtype=torch.float32)
    return time.perf_counter() - t0, out


def cpu_baseline(shape, n_sample, seed, reps=1, device=None):
    """The CPU baseline on a bounded sample; with `device`, the GPU layer runs
    the same sample (same weights and tokens, the other experts masked off
    through fused_moe's expert_mask) and its rel-L2 against the oracle's output
    is reported as the baseline's parity."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    s = cpu_sample_setup(shape, n_sample, seed)
    runs = [cpu_sample_run(s) for _ in range(reps)]
    sec, out_cpu = min(runs, key=lambda r: r[0])
    per_expert = sec / s["n"]
    tps = shape.M / (per_expert * s["active"])
    line = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"fp32 torch oracle (dequantise + matmul per expert) over {s['n']} of {s['active']} active "
                      f"experts of the M={shape.M} batch; seconds per expert x active experts = layer time"}
    if device is not None:
        from trials_b200 import moe

        g = lambda t: t.to(device)  # noqa: E731
        out_gpu = moe.fused_moe(g(s["hidden"]), g(s["w13_q"]), g(s["w2_q"]), g(s["tw"]), g(s["ids"]),
                                w1_scale=g(s["w13_s"]), w2_scale=g(s["w2_s"]),
                                expert_mask=g((s["emap"] >= 0).to(torch.int32)))
        line["parity"] = {"gpu_layer_vs_oracle_rel_l2": rel_l2(out_gpu.cpu(), out_cpu), "tol": 5e-3,
                          "what": "the GPU layer on the sampled experts against the oracle's output"}
    return line


def run_reference(args, shape, config):
    """The reference's torch path (restated by the oracle) on the host cores:
    each step runs the oracle over a bounded sample of the active experts of
    the whole job's tokens (all ranks' tokens at N > 1); ms_per_step is that
    measured time. The layer time is the measured seconds per expert times
    the active experts, which sets `value`."""
    import torch
    from dataclasses import replace

    rank, _, ws = dist_setup("gloo")
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    job = replace(shape, M=shape.M * ws)
    s = cpu_sample_setup(job, args.cpu_sample_experts, args.seed)
    for _ in range(args.warmup):
        cpu_sample_run(s)
    times = [cpu_sample_run(s)[0] for _ in range(args.steps)]
    step_s = sum(times) / len(times)
    per_expert = step_s / s["n"]
    layer_s = per_expert * s["active"]
    tps = job.M / layer_s
    sample = (f"fp32 torch oracle (restatement of the reference's torch path) over {s['n']} of {s['active']} "
              f"active experts of the job's {job.M} tokens per step; layer time = seconds per expert x active experts")
    line = {"metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config, "impl": "reference",
            "sample_scaling": {"experts_timed_per_step": s["n"], "active_experts": s["active"],
                               "measured_ms_per_step": step_s * 1e3, "layer_ms_estimated": layer_s * 1e3,
                               "tokens": job.M,
                               "note": "value = tokens / (ms_per_step / experts_timed_per_step x active_experts)"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------
CONFIG5_TOKENS = 8192  # expert-parallel configuration: tokens in total, split evenly over the ranks


def run_ep(args, shape, config):
    """N > 1: expert-parallel layer, E/N experts and M tokens per GPU, plus the
    parity and config5 records."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from trials_b200 import ep, moe, synth

    rank, local, ws = dist_setup("nccl")
    dev = torch.device("cuda", local)
    check = not args.no_parity
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=args.seed, device=dev)  # same weights on every rank
    hidden, tw, ids = layer_inputs(shape, shape.M, shape.hot_experts, args.seed + 1000 + rank, dev)
    M5 = CONFIG5_TOKENS // ws
    run5 = not args.no_config5 and M5 > 0
    if run5:
        h5, tw5, ids5 = layer_inputs(shape, M5, shape.hot_experts, args.seed + 2000 + rank, dev)
    # The single-GPU layer over all experts, on this rank's tokens: the parity reference.
    full = lambda h, w, i: moe.moe_decode_megakernel_full(h, L.w13, L.w13_scale, L.w2, L.w2_scale, w, i)  # noqa
    ref = full(hidden, tw, ids) if check else None
    ref5 = full(h5, tw5, ids5) if (check and run5) else None
    shards = [ep.shard_experts(t, rank, ws) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
    # config5 with 16 hot experts: the even split against hot-expert replication
    # (eplb_placement from the load of this batch's ids over all ranks; in
    # service the load would come from recent batches).
    run_hot = run5 and not args.no_eplb
    if run_hot:
        hh, htw, hids = layer_inputs(shape, M5, 16, args.seed + 5000 + rank, dev)
        parts = [torch.empty_like(hids) for _ in range(ws)]
        dist.all_gather(parts, hids)
        load = torch.bincount(torch.cat(parts).reshape(-1).long(), minlength=shape.E).cpu().numpy()
        spare = max(1, shape.E // (4 * ws))
        placement = ep.eplb_placement(load, ws, shape.E // ws + spare)
        placed = [ep.place_experts(t, placement, rank) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
        refh = full(hh, htw, hids) if check else None
    del L, full
    torch.cuda.empty_cache()
    model = ep.ExpertParallelMoE(*shards, num_experts=shape.E, rows_per_rank=shape.M, exchange=args.exchange)
    per = shape.E // ws

    def local_work(ids_rank):
        """(active local experts, local slots) of this rank over every rank's ids."""
        parts = [torch.empty_like(ids_rank) for _ in range(ws)]
        dist.all_gather(parts, ids_rank)
        glob = torch.cat(parts).reshape(-1)
        mine = glob[(glob >= rank * per) & (glob < (rank + 1) * per)]
        return int(torch.unique(mine).numel()), int(mine.numel())

    local_active, local_pairs = local_work(ids)

    def barrier():
        dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    clocks.start()

    def timed(m, h, w, i, steps, warmup, group):
        """Max over ranks of the mean step time, and of each stage's mean time."""
        for _ in range(warmup):
            m(h, w, i)
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        t0 = clocks.mark()
        start.record()
        for k in range(steps):
            m(h, w, i, events=evs[k])
        end.record()
        barrier()
        clocks.window(t0, clocks.mark(), group)
        ms = max_over_ranks(start.elapsed_time(end) / steps)
        stage_ms = {name: max_over_ranks(statistics.mean(evs[k][j].elapsed_time(evs[k][j + 1]) for k in range(steps)))
                    for j, name in enumerate(ep.ExpertParallelMoE.STAGES)}
        return ms, stage_ms

    ms, stage_ms = timed(model, hidden, tw, ids, args.steps, args.warmup, "main")
    errs = model.device_errors()
    # Ours per step: plan, pack (quantising on the way with the peer exchange; a
    # separate quant before it with NCCL), routing (which also waits for and
    # unpacks the received rows with the peer exchange when it runs on one CTA;
    # the unpack is a launch of its own otherwise), gather, the experts launch
    # (two for token-major tiles; two more for the heavy-expert list of a
    # mixed-list batch), top-k reduce, combine; routing is two launches from
    # 16,384 slots. The NCCL exchange adds its own all-to-all kernels, not
    # counted.
    from trials_b200 import _lib
    from trials_b200.stages import pick_tile_tokens

    def launches_per_step(M_rank):
        lib = _lib.lib()
        R = ws * M_rank  # received rows
        # the packed layer picks its tile from the slots expected on the rank
        tile = pick_tile_tokens(M_rank * shape.topk, per)
        heavy = lib.b200moe_heavy_rows(R, shape.topk, tile) > 0
        multi_route = lib.b200moe_route_scratch_ints(R * shape.topk, per) > 0 and not heavy
        n = 2 + (2 if multi_route else 1) + 1 + (2 if tile > 64 else 1) + (2 if heavy else 0) + 2
        if args.exchange == "peer":
            return n + (1 if multi_route else 0)
        return n + 2  # quant, unpack

    ep_launches = launches_per_step(shape.M)

    e2e = None
    if not args.no_e2e:
        t0 = clocks.mark()
        ms_copy, h2d, d2h = pipelined_e2e((hidden, ids, tw), lambda v: model(v[0], v[2], v[1]), (shape.M, shape.H),
                                     args.steps, args.warmup, barrier)
        clocks.window(t0, clocks.mark())
        ms_e2e = max_over_ranks(ms_copy)
        e2e = {"value": shape.M * ws / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d * ws,
               "d2h_bytes_per_step": d2h * ws, "ms_per_step": ms_e2e,
               "copies": "input and result copies on streams of their own, double-buffered: they overlap the neighbouring steps' layers"}

    other_x = "nccl" if args.exchange == "peer" else "peer"

    def parity(m, h, w, i, r):
        """This rank's output against the single-GPU layer, and against the
        other exchange form bit for bit; max / OR over ranks."""
        out = m(h, w, i).clone()
        other = ep.ExpertParallelMoE(*shards, num_experts=shape.E, rows_per_rank=m.cap, exchange=other_x)
        out_o = other(h, w, i)
        e = m.device_errors() | other.device_errors()
        other.close()
        rel = max_over_ranks(rel_l2(out, r))
        unequal = max_over_ranks(0.0 if torch.equal(out, out_o) else 1.0)
        e = int(max_over_ranks(float(e)))
        tol = 5e-3
        return {"reference": "single-GPU layer (moe_decode_megakernel_full) over all experts, same tokens",
                "rel_l2_max_over_ranks": rel, "tol": tol, f"bit_equal_{args.exchange}_vs_{other_x}": unequal == 0,
                "device_errors": e, "ok": rel <= tol and unequal == 0 and e == 0}

    par = parity(model, hidden, tw, ids, ref) if check else None

    c5 = None
    if run5:
        model5 = ep.ExpertParallelMoE(*shards, num_experts=shape.E, rows_per_rank=M5, exchange=args.exchange)
        ms5, st5 = timed(model5, h5, tw5, ids5, args.sweep_steps, 3, "config5")
        act5, pairs5 = local_work(ids5)
        act5, pairs5 = int(max_over_ranks(act5)), int(max_over_ranks(pairs5))
        peak, _ = measured_peaks()
        roof5 = experts_roofline(shape, act5, pairs5, st5["layer_packed"], peak)
        roof5["kernel"] = "layer_packed (the layer kernels on this rank's experts, incl. the wait for the dispatch)"
        c5 = {"workload": f"glm_ep_M{CONFIG5_TOKENS}_total", "tokens_total": M5 * ws, "tokens_per_gpu": M5,
              "value": M5 * ws / (ms5 / 1e3), "unit": "tokens/s", "ms_per_step": ms5, "steps": args.sweep_steps,
              "warmup": 3, "stage_ms": st5, "local_active_experts_max": act5, "local_pairs_max": pairs5,
              "roofline": roof5, "gpu_launches": launches_per_step(M5) * args.sweep_steps,
              "clocks": clocks.summary("config5")}
        if check:
            c5["parity"] = parity(model5, h5, tw5, ids5, ref5)
        errs |= model5.device_errors()
        model5.close()

    hot = None
    if run_hot:
        hot = {"workload": f"glm_ep_M{CONFIG5_TOKENS}_total_hot16", "tokens_total": M5 * ws, "tokens_per_gpu": M5,
               "router": "+2.0 on the logits of experts 0..15", "steps": args.sweep_steps, "warmup": 3}
        for name, w, pl in (("even_split", shards, None), ("eplb", placed, placement)):
            m = ep.ExpertParallelMoE(*w, num_experts=shape.E, rows_per_rank=M5, exchange=args.exchange, placement=pl)
            msh, sth = timed(m, hh, htw, hids, args.sweep_steps, 3, "config5")
            rec = {"ms_per_step": msh, "value": M5 * ws / (msh / 1e3), "unit": "tokens/s", "stage_ms": sth}
            if pl is not None:
                rec.update(slots_per_rank=pl.slots, max_replicas=pl.max_replicas,
                           replicated_experts=int((np.bincount(pl.phys_to_logical, minlength=shape.E) > 1).sum()))
            if check:
                out = m(hh, htw, hids)
                rel = max_over_ranks(rel_l2(out, refh))
                rec["parity"] = {"rel_l2_max_over_ranks": rel, "tol": 5e-3, "ok": rel <= 5e-3}
            errs |= m.device_errors()
            m.close()
            hot[name] = rec

    clk = clocks.stop()
    worst_active = int(max_over_ranks(local_active))
    if rank == 0:
        peak, peak_kind = measured_peaks()
        wbytes = worst_active * (synth.weight_bytes_per_expert(shape.H, shape.I) +
                                 synth.scale_bytes_per_expert(shape.H, shape.I))
        achieved = wbytes / (stage_ms["layer_packed"] / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": shape.M * ws / (ms / 1e3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8e4m3 (fp32 accumulate)", "data": "synthetic",
            "config": config, "stage_ms": stage_ms, "local_active_experts_max": worst_active,
            "roofline": {"kernel": "layer_packed (the five layer kernels on this rank's experts)", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} HBM copy bandwidth",
                         "algorithmic_bytes_per_launch": wbytes, "traffic": None},
            "gpu_launches": ep_launches * args.steps,
            "clocks": clk,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if par is not None:
            line["parity"] = par
        if c5 is not None:
            line["config5"] = c5
        if hot is not None:
            line["config5_hot16"] = hot
        if errs:
            line["device_errors"] = errs
        print(json.dumps(line), flush=True)
    model.close()
    dist.destroy_process_group()
    return 0


# The other single-GPU workloads of the benchmark set, measured on the same
# weights after the headline: (kind, tokens, hot experts).
SWEEP = (("decode", 128, 0), ("decode", 256, 0), ("decode", 512, 0), ("decode", 1024, 0), ("decode", 1024, 16),
         ("prefill", 2048, 0), ("prefill", 4096, 0), ("prefill", 8192, 0))


def ncu_traffic_ratio(name: str):
    """DRAM bytes over algorithmic bytes of a kernel, from a committed ncu
    summary of a small case (profiles/<name>.txt, line
    'dram_over_algorithmic: X'); scales a full-size launch's algorithmic
    bytes when the full workload is too large to capture."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_over_algorithmic:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


def run_sweep(args, shape, L, dev, clocks, peak):
    """Each SWEEP workload through the layer's launches (LayerPipeline, the
    kernels and order of b200moe_layer), CUDA events on their stream."""
    import torch

    from trials_b200 import stages, synth

    recs = []
    for kind, M, hot in SWEEP:
        # each workload starts from an idle GPU, not from the power state the previous one left
        time.sleep(0.5)
        h, tw, ids = layer_inputs(shape, M, hot, args.seed + 3000 + M + hot, dev)
        pipe = stages.LayerPipeline(M, shape.H, shape.I, shape.E, shape.topk, dev)
        w = (L.w13, L.w13_scale, L.w2, L.w2_scale)
        for _ in range(3):
            pipe.run(h, ids, tw, *w)
        steps = args.sweep_steps
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(pipe.stages) + 1)] for _ in range(steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0 = clocks.mark()
        start.record()
        for k in range(steps):
            pipe.run(h, ids, tw, *w, events=evs[k])
        end.record()
        torch.cuda.synchronize()
        clocks.window(t0, clocks.mark(), "sweep")
        ms = start.elapsed_time(end) / steps
        stage_ms = {n: statistics.mean(evs[k][i].elapsed_time(evs[k][i + 1]) for k in range(steps))
                    for i, n in enumerate(pipe.stages)}
        err = int(pipe.err.item())
        active = synth.active_experts(ids, shape.E)
        pairs = int(((ids >= 0) & (ids < shape.E)).sum().item())
        roof = experts_roofline(shape, active, pairs, stage_ms["experts"], peak)
        ratio = ncu_traffic_ratio("experts_tokmajor_small" if pipe.tile > 64 else "experts_swapab_small")
        roof["traffic"] = None if ratio is None else ratio * roof["algorithmic_bytes"]
        name = f"glm_{kind}_M{M}" + (f"_hot{hot}" if hot else "")
        recs.append({"workload": name, "tokens": M, "tile": pipe.tile, "ms_per_step": ms,
                     "value": M / (ms / 1e3), "unit": "tokens/s", "active_experts": active, "pairs": pairs,
                     "layer_hbm_gbs": layer_bytes(synth.glm(M), active, pairs) / (ms / 1e3) / 1e9,
                     "stage_ms": stage_ms, "roofline": roof, "device_error": err,
                     "heavy_experts_list": bool(pipe.heavy_rows),
                     "gpu_launches": pipe.launches * steps})
        del pipe, h, tw, ids
        torch.cuda.empty_cache()
    return {"steps": args.sweep_steps, "warmup": 3, "records": recs, "clocks": clocks.summary("sweep"),
            "pause_s_before_each": 0.5,
            "l2": "no flush: every step streams the active experts' weights (>= 8 GB)",
            "peaks": {"hbm_gbs": peak, "fp8_tflops": FP8_PEAK_TFLOPS}}


def run_router_record(args, shape, L, dev, clocks):
    """The headline batch from router logits (GLM routing: sigmoid + correction
    bias, top-k, renormalised, x2.5): the router as its own launch in front of
    the layer (select_experts, then the layer's launches) against the router
    inside routing's first launch (LayerPipeline.run_from_logits). Both give
    the same bits; the record has each one's step time and launches."""
    import torch

    from trials_b200 import moe, stages

    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 4000)
    logits = torch.randn(shape.M, shape.E, generator=g, device=dev)
    bias = torch.randn(shape.E, generator=g, device=dev) * 0.05
    router = {"scoring_func": "sigmoid", "correction_bias": bias, "renormalize": True, "routed_scaling_factor": 2.5}
    w = (L.w13, L.w13_scale, L.w2, L.w2_scale)
    sep = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, dev)
    fus = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, dev, router=router)

    def separate():
        tw, ids = moe.select_experts(logits, shape.topk, "sigmoid", bias, True, 2.5)
        return sep.run(L.hidden, ids, tw, *w)

    def fused():
        return fus.run_from_logits(L.hidden, logits, *w)

    rec = {"workload": f"glm_decode_M{shape.M}_from_router_logits",
           "router": "sigmoid + correction bias, top-8, renormalised, x2.5",
           "timing": "the two forms alternate over 3 rounds of sweep_steps steps; best round of each"}
    forms = (("separate_router", separate, 1), ("fused_router", fused, 0))
    for _, fn, _ in forms:
        for _ in range(3):
            fn()
    best = {name: float("inf") for name, _, _ in forms}
    for _ in range(3):
        for name, fn, _ in forms:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            t0 = clocks.mark()
            start.record()
            for _ in range(args.sweep_steps):
                fn()
            end.record()
            torch.cuda.synchronize()
            clocks.window(t0, clocks.mark(), "sweep")
            best[name] = min(best[name], start.elapsed_time(end) / args.sweep_steps)
    for name, _, router_launches in forms:
        launches = router_launches + sep.launches
        rec[name] = {"ms_per_step": best[name], "gpu_launches_per_step": launches, "steps": args.sweep_steps}
    rec["bit_equal"] = bool(torch.equal(separate(), fused()) and torch.equal(fus.topk_ids, moe.select_experts(
        logits, shape.topk, "sigmoid", bias, True, 2.5)[1]))
    rec["device_error"] = int(sep.err.item()) | int(fus.err.item())
    return rec


def run_whole_record(args, shape, L, dev, clocks):
    """The layer call (b200moe_layer) as one cooperative launch (routing,
    gather, both GEMM stages, top-k reduce) against the default separate
    launches, at 1, 64 and 128 tokens on the same weights. Each form is a CUDA
    graph of 10 calls (no host work timed); the forms alternate over 8 rounds
    of 3 replays; the record has each form's median step time, the launches
    per call and whether the outputs are equal bit for bit."""
    import statistics

    import torch

    from trials_b200 import _lib

    lib = _lib.lib()
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    recs = []
    prev = lib.b200moe_set_layer_launch(0)
    try:
        for M in (1, 64, 128):
            hidden, tw, ids = layer_inputs(shape, M, 0, args.seed + 5000 + M, dev)
            n = lib.b200moe_layer_workspace_size(M, shape.H, shape.I, shape.E, 0, shape.topk)
            forms = {1: "one_launch", 2: "separate"}
            ws = {m: torch.zeros(n, dtype=torch.uint8, device=dev) for m in forms}
            out = {m: torch.empty(M, shape.H, dtype=torch.bfloat16, device=dev) for m in forms}

            def call(m):
                _lib.check(lib.b200moe_layer(hidden.data_ptr(), M, shape.H, shape.I, shape.E, shape.topk,
                                             L.w13.data_ptr(), L.w13_scale.data_ptr(), L.w2.data_ptr(),
                                             L.w2_scale.data_ptr(), tw.data_ptr(), ids.data_ptr(), None, 0,
                                             out[m].data_ptr(), ws[m].data_ptr(), ws[m].numel(), st()), "layer")

            graphs, launches = {}, {}
            for m in forms:
                lib.b200moe_set_layer_launch(m)
                launches[m] = lib.b200moe_layer_launches(M, shape.H, shape.I, shape.E, 0, shape.topk)
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    for _ in range(3):
                        call(m)
                torch.cuda.current_stream().wait_stream(side)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(10):
                        call(m)
                graphs[m] = g
            times = {m: [] for m in forms}
            for rnd in range(8):
                for m in ((1, 2) if rnd % 2 == 0 else (2, 1)):
                    graphs[m].replay()
                    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    t0 = clocks.mark()
                    start.record()
                    for _ in range(3):
                        graphs[m].replay()
                    end.record()
                    torch.cuda.synchronize()
                    clocks.window(t0, clocks.mark(), "sweep")
                    times[m].append(start.elapsed_time(end) / 30)
            del graphs
            errs = [int(ws[m][:4].view(torch.int32).item()) for m in forms]
            rec = {"tokens": M, "bit_equal": bool(torch.equal(out[1], out[2])), "device_error": errs[0] | errs[1]}
            for m, name in forms.items():
                rec[name] = {"ms_per_step": statistics.median(times[m]), "gpu_launches_per_step": launches[m]}
            rec["one_launch_over_separate"] = statistics.median([a / b for a, b in zip(times[1], times[2])])
            recs.append(rec)
    finally:
        lib.b200moe_set_layer_launch(prev)
    return {"workload": "glm_decode_layer_call_one_launch_vs_separate",
            "timing": "CUDA graphs of 10 calls per form, 8 alternating rounds of 3 replays, medians",
            "default": "separate launches (b200moe_set_layer_launch(0))", "points": recs}


def run_ours(args, shape, config):
    import torch
    import torch.distributed as dist

    from trials_b200 import moe, stages, synth

    rank, local, ws = dist_setup("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=args.seed + rank, device=dev)
    active = synth.active_experts(L.topk_ids, shape.E)
    pairs = int(((L.topk_ids >= 0) & (L.topk_ids < shape.E)).sum().item())
    pipe = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, dev, tile_tokens=args.tile,
                                split=args.split, one_launch=args.layer_launch)
    args_run = (L.hidden, L.topk_ids, L.topk_weights, L.w13, L.w13_scale, L.w2, L.w2_scale)

    def barrier():
        if ws > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if ws == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing (value)
    for _ in range(args.warmup):
        pipe.run(*args_run)
    n_ev = len(pipe.stages) + 1
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n_ev)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    t0 = clocks.mark()
    start.record()
    for k in range(args.steps):
        pipe.run(*args_run, events=evs[k])
    end.record()
    barrier()
    clocks.window(t0, clocks.mark())
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    stage_ms = {name: statistics.mean(evs[k][i].elapsed_time(evs[k][i + 1]) for k in range(args.steps))
                for i, name in enumerate(pipe.stages)}
    err = int(pipe.err.item())
    if err:
        raise RuntimeError(f"device error word {err} after the timed steps")

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        t0 = clocks.mark()
        ms_copy, h2d, d2h = pipelined_e2e(
            (L.hidden, L.topk_ids, L.topk_weights),
            lambda v: moe.moe_decode_megakernel_full(v[0], L.w13, L.w13_scale, L.w2, L.w2_scale, v[2], v[1]),
            (shape.M, shape.H), args.steps, args.warmup, barrier)
        clocks.window(t0, clocks.mark())
        ms_e2e = max_over_ranks(ms_copy)
        e2e = {"value": shape.M * ws / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
               "copies": "input and result copies on streams of their own, double-buffered: they overlap the neighbouring steps' layers"}

    peak, peak_kind = measured_peaks()
    sweep = None
    if ws == 1 and not args.no_sweep:
        router_rec = run_router_record(args, shape, L, dev, clocks)  # before the power-capped prefill points
        whole_rec = run_whole_record(args, shape, L, dev, clocks)
        sweep = run_sweep(args, shape, L, dev, clocks, peak)
        sweep["router_fused"] = router_rec
        sweep["one_launch_layer"] = whole_rec
    clk = clocks.stop()

    # ---- CPU baseline (rank 0, one GPU only), with the GPU layer on the same sample
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(shape, args.cpu_sample_experts, args.seed, device=dev)

    if rank != 0:
        if ws > 1:
            dist.destroy_process_group()
        return 0
    hot = f"_hot{shape.hot_experts}" if shape.hot_experts else ""
    if "layer" in stage_ms:
        # Gather + quantise, both GEMM stages and the top-k reduce in one launch.
        k_name, k_bytes, k_ms = "layer (gather, grouped GEMM stages, top-k reduce; one launch)", \
            gemm1_bytes(shape, active, pairs) + gemm2_bytes(shape, active, pairs) + shape.M * shape.H * 2 * 2, \
            stage_ms["layer"]
        traffic_name = f"layer_glm_decode_m{shape.M}{hot}"
    elif "experts" in stage_ms:
        # Both GEMM stages in one launch (two launches for token-major tiles).
        k_name, k_bytes, k_ms = "experts (grouped GEMM, both stages)", \
            gemm1_bytes(shape, active, pairs) + gemm2_bytes(shape, active, pairs), stage_ms["experts"]
        traffic_name = f"experts_glm_decode_m{shape.M}{hot}"
    else:
        k_name, k_bytes, k_ms = "gemm1_silu (grouped GEMM stage 1)", gemm1_bytes(shape, active, pairs), \
            stage_ms["gemm1_silu"]
        traffic_name = f"gemm1_silu_glm_decode_m{shape.M}{hot}"
    achieved = k_bytes / (k_ms / 1e3) / 1e9
    launches = pipe.launches
    step_bytes = layer_bytes(shape, active, pairs)
    roof = {"kernel": k_name, "bound": "hbm", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_kind": f"{peak_kind} HBM copy bandwidth",
            "algorithmic_bytes_per_launch": k_bytes, "traffic": ncu_traffic(traffic_name)}
    if pipe.tile > 64 and "experts" in stage_ms:
        # Token-major tiles (prefill): a contraction, bounded by the tensor cores.
        flops = 2.0 * pairs * (2 * shape.I * shape.H + shape.H * shape.I)
        tf = flops / (stage_ms["experts"] / 1e3) / 1e12
        roof = {"kernel": "experts (token-major grouped GEMM stages, two launches)", "bound": "tensor",
                "achieved": tf, "peak": FP8_PEAK_TFLOPS, "unit": "TFLOP/s", "frac": tf / FP8_PEAK_TFLOPS,
                "peak_kind": "measured dense FP8 GEMM (torch._scaled_mm 8192^3 on this pool)",
                "algorithmic_flops_per_step": flops, "traffic": None}
        ratio = ncu_traffic_ratio("experts_tokmajor_small")
        if ratio is not None:  # small-case DRAM bytes over algorithmic bytes, scaled to this launch
            roof["traffic"] = ratio * (gemm1_bytes(shape, active, pairs) + gemm2_bytes(shape, active, pairs))
    line = {
        "metric": METRIC,
        "value": shape.M * ws / (ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8e4m3 (fp32 accumulate)",
        "data": "synthetic",
        "config": config,
        "hbm_gbs": step_bytes / (ms / 1e3) / 1e9,
        "hbm_frac": step_bytes / (ms / 1e3) / 1e9 / peak,
        "active_experts": active,
        "stage_ms": stage_ms,
        "roofline": roof,
        "gpu_launches": launches * args.steps,
        "clocks": clk,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if sweep is not None:
        line["sweep"] = sweep
    print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()
    return 0


def main(argv=None):
    args = parse_args(argv)
    from trials_b200 import synth

    shape = synth.glm(args.M, args.hot)
    if args.experts != shape.E:
        from dataclasses import replace

        shape = replace(shape, E=args.experts)
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    config = {"workload": f"glm_decode_M{args.M}" + (f"_hot{args.hot}" if args.hot else "") +
                          (f"_E{shape.E}" if shape.E != 256 else ""),
              "tokens_per_gpu": shape.M, "hidden": shape.H, "moe_intermediate": shape.I, "experts": shape.E,
              "topk": shape.topk, "router": "sigmoid top-k, renormalised",
              "quant": "e4m3 weights with fp32 128x128 block scales, 1x128 activation scales",
              "l2": "no flush: each step streams the active experts' fp8 weights (8.4-9.7 GB) >> 126 MB L2",
              "parallelism": "single GPU" if ws == 1 else
              f"expert parallel over {ws} GPUs: {shape.E // ws} experts and {shape.M} tokens per GPU, " +
              ("dispatch and combine stored by the kernels into peer memory over NVLink"
               if args.exchange == "peer" else "NCCL all-to-all dispatch and combine")}
    if args.impl == "reference":
        return run_reference(args, shape, config)
    if ws > 1:
        return run_ep(args, shape, config)
    return run_ours(args, shape, config)


if __name__ == "__main__":
    sys.exit(main())
