#!/usr/bin/env python
"""Benchmark of the decode hot path: KV-ring append + RoPE + attention, all 12 layers.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 1-6] [--impl ours|reference]

A *step* is one decode frame of every stream this GPU owns: all 12 layers'
append + RoPE + attention in one launch of the fused kernel (grid over layer x
item x head x chunk), through the C ABI (mb_decode_step).
Workloads:
  1            one stream/GPU, fp32 ring of 2048 slots with 300 filled, every step at
               position 300: the latency of one frame, L2 flushed before each timed step
  2 (default)  64 streams/GPU, 12 layers x 12 heads x 64, fp32 ring of 512 slots;
               positions 0..1499 (the ring wraps twice), repeated, reset between passes.
               With fewer timed steps than the job has (the driver's --steps 20),
               the whole job still runs, and the K timed steps sit at positions
               spread evenly over it, each timed alone with L2 flushed before it
  5            512 streams/GPU, bf16 ring of 4096 slots, live lengths U[1, 4096]
               from a seed, consecutive appends (streams shard by length at N > 1)
Weak scaling: every GPU runs its own streams; no collective on the decode path
(NCCL only for the barrier, the max-over-ranks timing and the report gather).

--impl reference times the reference algorithm on the host cores instead: the
CPU restatement in oracle/ (the reference is WGSL/TypeScript and cannot run
here), on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode frames/sec/GPU (all 12 layers' append+attn) and HBM GB/s vs roofline, 1/2/4/8 GPU"
H, HD = 12, 64
HID = H * HD
QKV = 3 * HID

CONFIGS = {
    1: dict(workload="config1: single-stream decode latency, 1 stream/GPU x 12 layers x 12 heads x 64, fp32 ring "
                     "capacity 2048 with 300 filled slots, q/k/v ~N(0,1), RoPE theta 10000 at position 300, one "
                     "append + attention per layer (every step appends position 300 again over the same 301-slot "
                     "window)",
            streams=1, layers=12, capacity=2048, dtype="f32", job_steps=None, steps=2000, warmup=20, position=300),
    2: dict(workload="config2: ring wraparound, 64 streams/GPU x 12 layers x 12 heads x 64, fp32 ring capacity "
                     "512, 1500 appends per stream (wraps twice), attention over the last <=512 positions every step",
            streams=64, layers=12, capacity=512, dtype="f32", job_steps=1500, steps=3000, warmup=30),
    3: dict(workload="config3: causal prefill, 32 streams x (188 prompt + 256 text = 444 positions) x 12 layers "
                     "x 12 heads x 64, fp16 ring storage (capacity 2048), fp32 accumulation, q/k/v ~ N(0, 0.5)",
            streams=32, layers=12, capacity=2048, dtype="f16", job_steps=None, steps=600, warmup=3, rows=444),
    4: dict(workload="config4: full 0.1B-class decoder decode step, 256 streams/GPU x 12 layers (hidden 768, 12 "
                     "heads x 64, FFN 3072), bf16 weights ~N(0,0.02) and bf16 ring capacity 2048, positions U[444,2048) "
                     "from seed 0; LN1 -> QKV GEMM -> append+RoPE+attention -> proj GEMM -> LN2 -> FFN per layer",
            streams=256, layers=12, capacity=2048, dtype="bf16", job_steps=None, steps=100, warmup=5, ffn=3072),
    5: dict(workload="config5: long-text serving, 512 streams/GPU x 12 layers x 12 heads x 64, bf16 ring capacity "
                     "4096, live lengths U[1,4096] from seed 0, consecutive appends",
            streams=512, layers=12, capacity=4096, dtype="bf16", job_steps=None, steps=200, warmup=5),
    6: dict(workload="local head: 256 streams/GPU, one frame = 17 sequential steps (one 768-wide layer, FFN 3072, "
                     "over a 17-slot ring; ln_f; 16 audio heads 768x1024 with greedy argmax and repetition penalty "
                     "1.2), bf16 weights ~N(0,0.02), tokens kept on the device",
            streams=256, layers=1, capacity=17, dtype="bf16", job_steps=None, steps=400, warmup=5, ffn=3072,
            codes=1024, channels=16),
}
LOCAL_METRIC = "local-head frames/sec/GPU (17 steps: layer + ln_f + audio head + penalised argmax)"


def _esize(dtype):
    return 4 if dtype == "f32" else 2


def window_bytes(L, esize, layers=12):
    """Algorithmic bytes of one stream-frame (all layers) at live window L:
    K,V window read 2*L*768*E + K,V append 2*768*E + q,k,v in and ctx out 4*768*4."""
    return layers * (2 * L * HID * esize + 2 * HID * esize + 4 * HID * 4)


# DRAM read + write per launch over the algorithmic bytes, from the full ncu capture
# of the fp32 decode kernel (one launch over all 12 layers of 8 streams, full
# 512-slot windows: 303.05 MB read + 6.28 MB written, mean of 2 launches, for
# 303.76 MB algorithmic; profiles/decode_kernel_f32_config2.md).  Traffic grows
# with the streams and the window, so a launch's traffic is its algorithmic bytes
# times this ratio.
DECODE_TRAFFIC_RATIO = {"f32": (303.05 + 6.28) / 303.76}
# slots per split-K chunk of the decode kernel (16 KB of K per chunk); windows longer
# than one chunk are combined by a second kernel launched behind the decode launch
DECODE_CHUNK_ROWS = {"f32": 64, "bf16": 128, "f16": 128}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s: the measured burst figure, else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device_index), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
            os.unlink(self.path)
        except Exception:
            return None
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        if not sm:
            return None
        mx = max(float(r[2]) for r in rows if len(r) >= 9)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons, "samples": len(sm)}


# ------------------------------------------------------------------ workloads
def config5_lengths(total, capacity, seed=0):
    return np.random.default_rng(seed).integers(1, capacity + 1, size=total)


def setup_ours(cfg, rank, world, device):
    """Rings, the qkv input pool in HBM, per-step positions."""
    import torch

    from mockbird_b200 import KvRing
    from mockbird_b200.scheduler import partition_streams

    n = cfg["streams"]
    ring = KvRing(layers=cfg["layers"], capacity=cfg["capacity"], streams=n, dtype=cfg["dtype"], wrap=True,
                  device=device.index, max_position=65536)
    g = torch.Generator(device=device)
    g.manual_seed(1234 + rank)
    set_bytes = cfg["layers"] * n * QKV * 4
    pool = max(2, -(-256 * 2**20 // set_bytes))  # > 2x L2 of distinct inputs
    qkv_pool = torch.randn(pool, cfg["layers"], n, QKV, generator=g, device=device)
    out = torch.empty(cfg["layers"], n, HID, device=device)
    streams = torch.arange(n, dtype=torch.int32, device=device)
    info = {"qkv_pool_sets": pool}
    if cfg["job_steps"] is not None:  # config 2: everyone at the same position
        lengths0 = None
        shard_ids = partition_streams(n * world, world)[rank].streams
        if cfg.get("start") is not None:  # steady state: the C positions before `start` are written
            C = cfg["capacity"]
            kv = torch.randn(2, H, C, HD, generator=g, device=device).to(ring.torch_dtype)
            for layer in range(cfg["layers"]):
                for i in range(n):
                    ring.ring_write(layer, i, cfg["start"] - C, kv[0], kv[1])
            torch.cuda.synchronize(device)
    else:  # config 5: per-stream live lengths, length-balanced shards
        total = n * world
        all_len = config5_lengths(max(total, 4096), cfg["capacity"])[:total]
        shard_ids = partition_streams(total, world, all_len)[rank].streams
        lengths0 = all_len[shard_ids].astype(np.int64)
        fill_lengths(ring, lengths0, cfg["layers"], g, device)
    info["global_streams"] = n * world
    info["shard"] = [int(shard_ids.min()), int(shard_ids.max())] if len(shard_ids) else []
    return ring, qkv_pool, out, streams, lengths0, info


def fill_lengths(ring, lengths0, layers, gen, device):
    """Config 5's starting rings: positions 0..L-2 of every stream filled with
    N(0,1) K/V (the same rows for all layers), every other slot empty."""
    import torch

    ring.reset()
    for i, L in enumerate(lengths0):
        if L <= 1:
            continue
        kv = torch.randn(2, H, int(L) - 1, HD, generator=gen, device=device).to(ring.torch_dtype)
        for layer in range(layers):
            ring.ring_write(layer, i, 0, kv[0], kv[1])
    torch.cuda.synchronize(device)


def positions_for(cfg, step, n, lengths0):
    """Host positions of every stream at `step` (a step of the job)."""
    if lengths0 is None:
        if cfg.get("start") is not None:
            return np.full(n, cfg["start"] + step, np.int32)
        return np.full(n, step % cfg["job_steps"], np.int32)
    return (lengths0 - 1 + step).astype(np.int32)


def live_len(pos, capacity):
    return np.minimum(pos + 1, capacity)


def sampled_positions(job_steps, k):
    """K positions spread evenly over a job of `job_steps` steps: step t at
    floor((t + 1/2) * job_steps / K), so the timed windows follow the job's own mix."""
    return [int((t + 0.5) * job_steps / k) for t in range(k)]


L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def run_ours(args, cfg, rank, world, device):
    import torch

    from mockbird_b200.scheduler import max_over_ranks

    ring, qkv_pool, out, streams, lengths0, info = setup_ours(cfg, rank, world, device)
    n, L, C = cfg["streams"], cfg["layers"], cfg["capacity"]
    K, W = args.steps, args.warmup
    es = _esize(cfg["dtype"])
    job = lengths0 is None and cfg.get("start") is None  # config 2's 1500-frame job
    J = cfg["job_steps"]
    # Sampled: fewer timed steps than the job has.  The whole job runs (so every
    # ring holds exactly the job's state), and only K steps spread evenly over it
    # are timed, each with its own event pair and with L2 flushed before it.
    sampled = job and K < J
    if sampled:
        timed = sampled_positions(J, K)
        pos_host = np.stack([positions_for(cfg, t, n, None) for t in range(J)])
    else:
        pos_host = np.stack([positions_for(cfg, t, n, lengths0) for t in range(W + K)])
        if job:  # warm-up 0..W-1, then the job from 0
            pos_host[W:] = np.stack([positions_for(cfg, t, n, None) for t in range(K)])
        timed = list(range(W, W + K))
    pos_dev = torch.from_numpy(pos_host).to(device)
    algo_bytes = sum(float(window_bytes(live_len(pos_host[t].astype(np.int64), C), es, L).sum()) for t in timed)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device) if sampled else None

    def step(t):
        if job and not sampled and t >= W and (t - W) % J == 0:
            ring.reset()  # a new pass of the 1500-frame job starts from an empty ring
        ring.decode_step(streams, pos_dev[t], qkv_pool[t % qkv_pool.shape[0]], out)

    for t in range(W):
        step(t)
    ring.sync()
    if job:
        ring.reset()
    dist = _dist()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    stream = torch.cuda.current_stream(device)
    if sampled:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in timed]
        k = 0
        for t in range(J):
            if k < K and t == timed[k]:
                flush.zero_()
                evs[k][0].record(stream)
                step(t)
                evs[k][1].record(stream)
                k += 1
            else:
                step(t)
        torch.cuda.synchronize(device)
        ms = sum(a.elapsed_time(b) for a, b in evs)
    else:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for t in range(W, W + K):
            step(t)
        ev1.record(stream)
        torch.cuda.synchronize(device)
        ms = ev0.elapsed_time(ev1)
    if dist:
        dist.barrier()
    ring.sync()
    ms_max = max_over_ranks(ms, device if dist else None)
    launches = K  # mb_decode_step: one decode launch covers every layer of the step
    kernels = 2 * K if C > DECODE_CHUNK_ROWS[cfg["dtype"]] else K  # + the split-K combine behind each

    # ---- end to end through the host-array C ABI call (pinned buffers), copies timed
    e2e = None
    if not args.no_e2e and cfg.get("start") is None:
        sets = 2
        host_qkv = torch.empty(sets, L, n, QKV, dtype=torch.float32).pin_memory()
        for i in range(sets):
            host_qkv[i].copy_(qkv_pool[i])
        host_out = torch.empty(L, n, HID, dtype=torch.float32).pin_memory()
        ids = np.arange(n, dtype=np.int32)
        if lengths0 is None:
            ring.reset()
        else:  # config 5: the starting rings again and the warm-up replayed, so the
            # e2e steps run the timed region's positions over the same windows
            gen = torch.Generator(device=device)
            gen.manual_seed(5678 + rank)
            fill_lengths(ring, lengths0, L, gen, device)
            for t in range(W):
                step(t)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        if sampled:  # the same K job positions through the host call; the other steps on the device
            e2e_s, k = 0.0, 0
            for t in range(J):
                if k < K and t == timed[k]:
                    flush.zero_()
                    stream.synchronize()
                    t0 = time.perf_counter()
                    ring.decode_step_host(ids, pos_host[t], host_qkv[t % sets], host_out)
                    e2e_s += time.perf_counter() - t0
                    k += 1
                else:
                    step(t)
            torch.cuda.synchronize(device)
        else:
            t0 = time.perf_counter()
            for t in range(K):
                if lengths0 is None and t > 0 and t % J == 0:
                    ring.reset()
                pos = positions_for(cfg, t, n, None) if lengths0 is None else pos_host[W + t]
                ring.decode_step_host(ids, pos, host_qkv[t % sets], host_out)
            torch.cuda.synchronize(device)
            e2e_s = time.perf_counter() - t0
        e2e_s = max_over_ranks(e2e_s, device if dist else None)
        e2e = {"value": world * n * K / e2e_s, "unit": "frames/s",
               "h2d_bytes_per_step": int(L * n * QKV * 4 + 2 * n * 4),
               "d2h_bytes_per_step": int(L * n * HID * 4),
               "steps": K, "api": "mb_decode_step_host (C ABI, pinned host buffers, blocking per step)"
               + ("; the same K sampled job positions, wall clock per call, L2 flushed before each" if sampled
                  else "")}
        if sampled:
            # The engine's own call shape as well: DecodeRunner.runLayer hands one
            # layer's qkv rows to the KV path at a time, so a frame is 12 blocking
            # host-array calls (mb_append_attend_host), the same K job positions.
            ring.reset()
            if dist:
                dist.barrier()
            torch.cuda.synchronize(device)
            lay_s, k = 0.0, 0
            for t in range(J):
                if k < K and t == timed[k]:
                    flush.zero_()
                    stream.synchronize()
                    t0 = time.perf_counter()
                    for layer in range(L):
                        ring.append_attend_host(layer, ids, pos_host[t], host_qkv[t % sets][layer],
                                                host_out[layer])
                    lay_s += time.perf_counter() - t0
                    k += 1
                else:
                    step(t)
            torch.cuda.synchronize(device)
            lay_s = max_over_ranks(lay_s, device if dist else None)
            e2e["per_layer_calls"] = {
                "value": round(world * n * K / lay_s, 1), "unit": "frames/s",
                "h2d_bytes_per_step": int(L * (n * QKV * 4 + 2 * n * 4)), "d2h_bytes_per_step": int(L * n * HID * 4),
                "api": "12 x mb_append_attend_host per frame (one blocking host-array call per layer, the shape "
                       "of DecodeRunner.runLayer), the same K sampled job positions, wall clock, L2 flushed "
                       "before each frame"}
    clk = clocks.stop()

    value = world * n * K / (ms_max / 1e3)
    peak, peak_kind = peaks()
    achieved = algo_bytes / (ms / 1e3) / 1e9  # this rank's algorithmic bytes over its own device time
    ratio = DECODE_TRAFFIC_RATIO.get(cfg["dtype"])
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": round(algo_bytes / launches * ratio) if ratio else None,
                "traffic_source": "ncu capture of a smaller case scaled by algorithmic bytes per launch "
                                  "(profiles/decode_kernel_f32_config2.md)" if ratio else None,
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "kernel": "decode_kernel<fused append+RoPE+split-K attention>, all 12 layers of a step in one launch",
                "algorithmic_bytes_per_launch": algo_bytes / launches,
                "avg_launch_us": ms * 1e3 / launches,
                "avg_launch_us_note": "per decode launch, including the split-K combine launched behind it",
                "timing": ("CUDA events around each timed step on the launching stream (sum over the K steps); "
                           if sampled else "CUDA events over the timed region on the launching stream; ")
                + "every launch timed is this kernel, so avg launch = timed time / launches (launch gaps included)"}
    if sampled:
        timing_note = (f"{K} of the job's {J} steps timed, at positions floor((t + 1/2) * {J} / {K}) "
                       f"({timed[0]}, {timed[1] if K > 1 else ''} ... {timed[-1]}); the other steps run untimed "
                       f"in order, so each timed step sees the job's own ring; L2 flushed (256 MB write) before "
                       f"each timed step")
    elif job:
        timing_note = f"{K} consecutive steps of the job (positions t mod {J}, reset between passes)"
    else:
        timing_note = f"{K} consecutive steps"
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "frames/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded N(0,1) q/k/v; random ring contents)",
        "config": {"workload": cfg["workload"], "streams_per_gpu": n, "global_streams": info["global_streams"],
                   "layers": L, "heads": H, "head_dim": HD, "capacity": C, "storage": cfg["dtype"],
                   "parallelism": f"stream-sharded x{world} (no collective on the decode path)",
                   "timed_steps": timing_note,
                   "mean_window": round(float(np.mean([live_len(pos_host[t].astype(np.int64), C).mean()
                                                       for t in timed])), 1),
                   "l2": (f"L2 flushed before every timed step; ~{algo_bytes / K / 1e9:.2f} GB of K/V windows per "
                          "timed step" if sampled else
                          "inputs larger than L2: every step streams the live K/V windows "
                          f"(~{algo_bytes / K / 1e9:.2f} GB/step) plus {info['qkv_pool_sets']} rotating qkv sets"),
                   "value_per_gpu": round(value / world, 1)},
        "roofline": roofline, "e2e": e2e, "gpu_launches": kernels, "clocks": clk,
    }
    return result, ring


def run_single(args, cfg, rank, world, device):
    """Config 1: the latency of one frame of one stream (12 layers' append +
    RoPE + attention at position 300 over a 2048-slot ring holding positions
    0..299).  Every step appends position 300 again, so every step attends the
    same 301-row window; L2 is flushed before each timed step and each step is
    timed alone with its own event pair."""
    import torch

    from mockbird_b200 import KvRing
    from mockbird_b200.scheduler import max_over_ranks

    n, L, C, P = cfg["streams"], cfg["layers"], cfg["capacity"], cfg["position"]
    K, W = args.steps, args.warmup
    ring = KvRing(layers=L, capacity=C, streams=n, dtype=cfg["dtype"], wrap=True, device=device.index,
                  max_position=65536)
    g = torch.Generator(device=device)
    g.manual_seed(rank)
    for i in range(n):
        kv = torch.randn(2, L, H, P, HD, generator=g, device=device).to(ring.torch_dtype)
        for layer in range(L):
            ring.ring_write(layer, i, 0, kv[0, layer], kv[1, layer])
    sets = 4
    qkv = torch.randn(sets, L, n, QKV, generator=g, device=device)
    out = torch.empty(L, n, HID, device=device)
    streams = torch.arange(n, dtype=torch.int32, device=device)
    pos = torch.full((n,), P, dtype=torch.int32, device=device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    es = _esize(cfg["dtype"])
    algo = float(window_bytes(live_len(np.full(n, P, np.int64), C), es, L).sum())

    for t in range(W):
        ring.decode_step(streams, pos, qkv[t % sets], out)
    dist = _dist()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for t in range(K):
        flush.zero_()
        evs[t][0].record(stream)
        ring.decode_step(streams, pos, qkv[t % sets], out)
        evs[t][1].record(stream)
    torch.cuda.synchronize(device)
    per = sorted(a.elapsed_time(b) for a, b in evs)
    ms = sum(per)
    # the same steps back to back, L2 warm (the window stays resident between frames)
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for t in range(K):
        ring.decode_step(streams, pos, qkv[t % sets], out)
    w1.record(stream)
    torch.cuda.synchronize(device)
    warm_ms = w0.elapsed_time(w1)

    e2e = None
    if not args.no_e2e:
        host_qkv = torch.empty(sets, L, n, QKV, dtype=torch.float32).pin_memory()
        host_qkv.copy_(qkv.cpu())
        host_out = torch.empty(L, n, HID, dtype=torch.float32).pin_memory()
        ids, hpos = np.arange(n, dtype=np.int32), np.full(n, P, np.int32)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(device)
        e2e_s = lay_s = 0.0
        for t in range(K):
            flush.zero_()
            stream.synchronize()
            t0 = time.perf_counter()
            ring.decode_step_host(ids, hpos, host_qkv[t % sets], host_out)
            e2e_s += time.perf_counter() - t0
        for t in range(K):  # the engine's call shape: one blocking host-array call per layer
            flush.zero_()
            stream.synchronize()
            t0 = time.perf_counter()
            for layer in range(L):
                ring.append_attend_host(layer, ids, hpos, host_qkv[t % sets][layer], host_out[layer])
            lay_s += time.perf_counter() - t0
        e2e_s = max_over_ranks(e2e_s, device if dist else None)
        lay_s = max_over_ranks(lay_s, device if dist else None)
        e2e = {"value": round(world * n * K / e2e_s, 1), "unit": "frames/s",
               "h2d_bytes_per_step": int(L * n * QKV * 4 + 2 * n * 4), "d2h_bytes_per_step": int(L * n * HID * 4),
               "steps": K, "latency_us": round(e2e_s / K * 1e6, 2),
               "api": "mb_decode_step_host (C ABI, pinned host buffers, blocking per step), wall clock per call, "
                      "L2 flushed before each",
               "per_layer_calls": {
                   "value": round(world * n * K / lay_s, 1), "unit": "frames/s",
                   "latency_us": round(lay_s / K * 1e6, 2),
                   "h2d_bytes_per_step": int(L * (n * QKV * 4 + 2 * n * 4)),
                   "d2h_bytes_per_step": int(L * n * HID * 4),
                   "api": "12 x mb_append_attend_host per frame (one blocking host-array call per layer, the "
                          "shape of DecodeRunner.runLayer), wall clock, L2 flushed before each frame"}}
    clk = clocks.stop()
    ms_max = max_over_ranks(ms, device if dist else None)
    value = world * n * K / (ms_max / 1e3)
    peak, peak_kind = peaks()
    achieved = algo * K / (ms / 1e3) / 1e9
    chunks = -(-min(P + 1, C) // DECODE_CHUNK_ROWS[cfg["dtype"]])
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": None,
                "traffic_note": "not captured for this case: after each flush the 22 MB window comes from HBM "
                                "once; ncu would add the flush's write-back to the flush kernel, not to this one",
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "kernel": f"decode_kernel over {L} layers x {H} heads x {chunks} chunks = {L * H * chunks} CTAs, "
                          "then the split-K combine",
                "algorithmic_bytes_per_launch": algo, "avg_launch_us": round(ms * 1e3 / K, 3),
                "avg_launch_us_note": "per step: the decode launch and the combine behind it, each step timed "
                                      "alone (CUDA events on the launching stream) after an L2 flush",
                "bound_note": "a single frame moves 22 MB, a few microseconds of HBM time; the launch and "
                              "the two kernels' fixed latencies dominate it"}
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "frames/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded N(0,1) q/k/v and ring rows)",
        "config": {"workload": cfg["workload"], "streams_per_gpu": n, "global_streams": n * world, "layers": L,
                   "heads": H, "head_dim": HD, "capacity": C, "storage": cfg["dtype"], "position": P,
                   "parallelism": f"stream-sharded x{world} (no collective on the decode path)",
                   "timed_steps": f"{K} steps, each timed alone with its own event pair",
                   "l2": "L2 flushed (256 MB write) before every timed step",
                   "latency_us": {"mean": round(ms / K * 1e3, 3), "p50": round(per[K // 2] * 1e3, 3),
                                  "p99": round(per[min(K - 1, (99 * K) // 100)] * 1e3, 3)},
                   "warm_l2_back_to_back_us": round(warm_ms / K * 1e3, 3),
                   "value_per_gpu": round(value / world, 1)},
        "roofline": roofline, "e2e": e2e, "gpu_launches": 2 * K if chunks > 1 else K, "clocks": clk,
    }
    return result, ring


def run_cpu_single(cfg, steps, budget_s=None):
    """Config 1 on the host cores: the oracle's append_attend (the reference's
    ROPE_SPLIT_CACHE + ATTENTION_* restated) for one stream at position 300 over
    positions 0..299, all 12 layers per frame, OpenMP over the 12 heads."""
    cores = use_all_host_threads()
    import oracle

    L, C, P = cfg["layers"], cfg["capacity"], cfg["position"]
    ring = oracle.Ring(layers=L, streams=1, heads=H, capacity=C, dtype=cfg["dtype"], wrap=True, max_position=8192)
    rng = np.random.default_rng(0)
    ring.kv_view()[:, 0, :, :, :P] = rng.standard_normal((L, 2, H, P, HD)).astype(np.float32)
    ring.slot_pos[:, 0, :P] = np.arange(P)
    qkv = rng.standard_normal((4, L, 1, QKV)).astype(np.float32)
    ids, pos = np.zeros(1, np.int32), np.full(1, P, np.int32)
    for t in range(3):
        for layer in range(L):
            ring.append_attend(layer, ids, pos, qkv[t % 4, layer])
    t0 = time.perf_counter()
    done = 0
    for t in range(steps):
        for layer in range(L):
            ring.append_attend(layer, ids, pos, qkv[t % 4, layer])
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done / dt, 2), "unit": "frames/s", "cores": cores, "kind": "port",
            "latency_us": round(dt / done * 1e6, 1),
            "sample": f"{done} frames of the one stream at position {P}, all {L} layers per frame, oracle/oracle.c "
                      f"fp32 mirror of the WGSL kernels, OpenMP over the heads, {dt:.1f} s"}


def _dist():
    try:
        import torch.distributed as dist
        return dist if dist.is_initialized() else None
    except Exception:
        return None


# ------------------------------------------------------------------ config 3: causal prefill
def prefill_flops(rows, streams, layers=12):
    """Causal QK^T + PV FLOPs: 4 * 64 * 12 * S(S+1)/2 per layer per stream."""
    return 4.0 * HD * H * rows * (rows + 1) / 2 * streams * layers


def run_prefill(args, cfg, rank, world, device):
    """A step = the 12-layer prefill of every stream on this GPU (12 mb_prefill calls)."""
    import torch

    from mockbird_b200 import KvRing
    from mockbird_b200.scheduler import max_over_ranks

    n, L, C, S = cfg["streams"], cfg["layers"], cfg["capacity"], cfg["rows"]
    ring = KvRing(layers=L, capacity=C, streams=n, dtype=cfg["dtype"], wrap=True, device=device.index)
    g = torch.Generator(device=device)
    g.manual_seed(4321 + rank)
    qkv = torch.randn(L, n, S, QKV, generator=g, device=device) * 0.5  # 1.57 GB: one step's inputs
    out = torch.empty(n, S, HID, device=device)
    streams = torch.arange(n, dtype=torch.int32, device=device)
    for _ in range(args.warmup):
        for layer in range(L):
            ring.prefill(layer, streams, qkv[layer], out)
    ring.sync()
    dist = _dist()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        for layer in range(L):
            ring.prefill(layer, streams, qkv[layer], out)
    ev1.record(stream)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ring.sync()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, device if dist else None)
    flops = prefill_flops(S, n, L) * args.steps
    tpeak, tkind = tensor_peak()
    achieved = flops / (ms / 1e3) / 1e12
    # The step's compulsory HBM traffic per row and layer: q, k, v read (fp32),
    # K and V written to the ring (storage type), the context written (fp32).  At
    # config 3 that is ~218 MB per layer (~34 us at the measured copy bandwidth)
    # against ~6 us of tensor work at the bf16 peak: the step is HBM-bound, and
    # the tensor pipe's share is reported beside it.
    es = _esize(cfg["dtype"])
    hbm_bytes = float(n * S * L * (QKV * 4 + 2 * HID * es + HID * 4)) * args.steps
    hpeak, hkind = peaks()
    hbm_achieved = hbm_bytes / (ms / 1e3) / 1e9
    result = {
        "metric": "causal prefill attention TFLOP/s (config 3; RoPE+cache write and attention, all 12 layers)",
        "value": round(world * flops / (ms_max / 1e3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded N(0, 0.5) q/k/v)",
        "config": {"workload": cfg["workload"], "streams_per_gpu": n, "rows": S, "layers": L,
                   "l2": "inputs larger than L2: 1.57 GB of qkv per step",
                   "positions_per_s": round(world * n * S * args.steps / (ms_max / 1e3), 1)},
        "roofline": {"bound": "hbm", "achieved": round(hbm_achieved, 1), "peak": hpeak, "unit": "GB/s",
                     "frac": round(hbm_achieved / hpeak, 4), "traffic": None,
                     "peak_source": f"{hkind} hbm_gbs (MEASURED_PEAKS.json)",
                     "algorithmic_bytes_per_step": hbm_bytes / args.steps,
                     "bytes": "per row and layer: q, k, v read (fp32), K and V written to the ring, context written "
                              "(fp32)",
                     "tensor": {"achieved": round(achieved, 2), "peak": tpeak, "unit": "TFLOP/s",
                                "frac": round(achieved / tpeak, 4), "peak_source": f"{tkind} bf16_tflops (burst)",
                                "flops": "causal QK^T + PV only"},
                     "timing": "CUDA events over the whole prefill calls (RoPE/cache kernel + attention kernel)"},
        "gpu_launches": 2 * L * args.steps, "clocks": clk, "e2e": None,
    }
    return result, ring


# ------------------------------------------------------------------ config 4: the full decoder step
def decoder_weights(layers, h, ffn, seed=0):
    """N(0, 0.02) weights in the published graph's order, LayerNorm gains 1."""
    from mockbird_b200.engine import Decoder

    per = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * ffn + ffn + ffn * h + h
    w = (np.random.default_rng(seed).standard_normal(Decoder.weight_count(layers, h, ffn)) * 0.02).astype(np.float32)
    for l in range(layers):
        b = l * per
        w[b:b + h] = 1.0
        w[b + 2 * h + 3 * h * h + 3 * h + h * h + h: b + 2 * h + 3 * h * h + 3 * h + h * h + 2 * h] = 1.0
    w[layers * per: layers * per + h] = 1.0
    return w


def config4_positions(n, capacity, seed=0):
    return np.random.default_rng(seed).integers(444, capacity, size=n)


def run_decoder(args, cfg, rank, world, device):
    import torch

    from mockbird_b200 import KvRing
    from mockbird_b200.engine import Decoder
    from mockbird_b200.scheduler import max_over_ranks

    n, L, C, F = cfg["streams"], cfg["layers"], cfg["capacity"], cfg["ffn"]
    ring = KvRing(layers=L, capacity=C, streams=n, dtype=cfg["dtype"], wrap=True, device=device.index)
    dec = Decoder(ring, decoder_weights(L, HID, F), F)
    # the step's kernel chains: two half batches from 128 items up (MOCKBIRD_DECODER_SPLIT=0: one)
    chains = 2 if n >= 128 and os.environ.get("MOCKBIRD_DECODER_SPLIT", "1") != "0" else 1
    pos0 = config4_positions(n * world, C)[rank * n:(rank + 1) * n].astype(np.int64)

    def fill():
        """The starting rings: positions 0..p0-1 of every stream in every layer
        (seeded, so a refill restores the same contents); returns the generator."""
        gen = torch.Generator(device=device)
        gen.manual_seed(77 + rank)
        ring.reset()
        for i, p0 in enumerate(pos0):
            kv = torch.randn(2, H, int(p0), HD, generator=gen, device=device).to(ring.torch_dtype)
            for layer in range(L):
                ring.ring_write(layer, i, 0, kv[0], kv[1])
        torch.cuda.synchronize(device)
        return gen

    g = fill()
    K, W = args.steps, args.warmup
    pos_dev = torch.from_numpy(np.stack([(pos0 + t).astype(np.int32) for t in range(W + K)])).to(device)
    streams = torch.arange(n, dtype=torch.int32, device=device)
    rows = torch.randn(8, n, HID, generator=g, device=device)  # embedded rows, rotating
    hidden = torch.empty(n, HID, device=device)
    for t in range(W):
        hidden.copy_(rows[t % 8])
        dec.step(streams, pos_dev[t], hidden)
    ring.sync()
    dist = _dist()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for t in range(W, W + K):
        hidden.copy_(rows[t % 8])
        dec.step(streams, pos_dev[t], hidden)
    ev1.record(stream)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ring.sync()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, device if dist else None)
    # e2e: through mb_decoder_step_host, the call DecodeRunner.globalStep makes --
    # the embedded rows from pinned host memory in, the ln_f rows back into the
    # same buffer, one synchronisation per step (each step's output row is the
    # next step's input row).  The rings are restored and the warm-up replayed
    # first, so the e2e steps run the timed region's positions over the same windows.
    host_rows = torch.empty(n, HID).pin_memory()
    host_rows.copy_(rows[0].cpu())
    ids = np.arange(n, dtype=np.int32)
    pos_host = np.stack([(pos0 + t).astype(np.int32) for t in range(W + K)])
    fill()
    for t in range(W):
        hidden.copy_(rows[t % 8])
        dec.step(streams, pos_dev[t], hidden)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for t in range(W, W + K):
        dec.step_host(ids, pos_host[t], host_rows)
    e2e_s = max_over_ranks(time.perf_counter() - t0, device if dist else None)
    es = _esize(cfg["dtype"])
    live = np.minimum(pos0[None, :] + np.arange(W, W + K)[:, None] + 1, C)
    kv_bytes = float((2 * live * HID * es + 2 * HID * es).sum()) * L
    w_bytes = L * (HID * 3 * HID + HID * HID + 2 * HID * F) * 2.0 * K
    act_bytes = L * n * K * 4.0 * (4 * HID)
    algo = kv_bytes + w_bytes + act_bytes
    peak, peak_kind = peaks()
    achieved = algo / (ms / 1e3) / 1e9
    value = world * n * K / (ms_max / 1e3)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": "frames/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": "synthetic (seeded N(0,1) rows and K/V, N(0,0.02) weights)",
        "config": {"workload": cfg["workload"], "streams_per_gpu": n, "global_streams": n * world, "layers": L,
                   "capacity": C, "ffn": F, "parallelism": f"stream-sharded x{world} (no collective on the decode path)",
                   "l2": f"inputs larger than L2: ~{kv_bytes / K / 1e9:.1f} GB of K/V windows per step",
                   "value_per_gpu": round(value / world, 1),
                   "gemms": "this library's tcgen05 GEMMs (bias, residual and GELU in their epilogues); LayerNorm and "
                            "the attention are this library's kernels too"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "kernel": "whole decoder step (decode_kernel dominates: K/V windows are ~98% of the bytes)",
                     "timing": "CUDA events over the timed region; algorithmic bytes = K/V windows + appends + "
                               "weights + activations"},
        "e2e": {"value": round(world * n * K / e2e_s, 1), "unit": "frames/s",
                "h2d_bytes_per_step": n * HID * 4, "d2h_bytes_per_step": n * HID * 4,
                "api": "mb_decoder_step_host (C ABI): the embedded rows from pinned host memory in, the ln_f rows "
                       "back to it, one synchronisation per step"},
        "gpu_launches": K * chains * (L * 8 + 1),
        "clocks": clk,
    }
    result["gpu_launches_note"] = ("8 of this library's kernels per layer (LN1, QKV GEMM, attention, its split-K "
                                   "combine, c_proj GEMM, LN2, fc_in GEMM + GELU, fc_out GEMM) + ln_f, per "
                                   f"half-batch chain ({chains} chain{'s' if chains > 1 else ''}: a step of >= 128 "
                                   "items runs as two, on two CUDA streams)")
    dec.dispose()
    return result, ring


def use_all_host_threads():
    """The CPU legs run on every host thread this process may use.  torchrun sets
    OMP_NUM_THREADS=1 in its workers, and the oracle's OpenMP runtime reads that
    variable when it is first loaded, so it is set here, before that load."""
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    os.environ["OMP_NUM_THREADS"] = str(cores)
    return cores


def run_cpu_decoder(cfg, steps, sample_streams=2, budget_s=None):
    """The reference's decode step (ref-decode.mjs decodeStep restated by the oracle) on the host cores."""
    use_all_host_threads()
    import oracle

    n, L, C, F = sample_streams, cfg["layers"], cfg["capacity"], cfg["ffn"]
    ring = oracle.Ring(layers=L, streams=n, heads=H, capacity=C, dtype=cfg["dtype"], wrap=True, max_position=4096)
    w = decoder_weights(L, HID, F)
    rng = np.random.default_rng(5)
    pos0 = config4_positions(n, C)
    kvv = ring.kv_view()
    for s_ in range(n):
        p0 = int(pos0[s_])
        rows = rng.standard_normal((2, H, p0, HD)).astype(np.float32)
        kvv[:, s_, :, :, :p0] = ((rows.view(np.uint32) >> 16).astype(np.uint16))[None]
        ring.slot_pos[:, s_, :p0] = np.arange(p0)
    x = rng.standard_normal((n, HID)).astype(np.float32)
    t0 = time.perf_counter()
    done = 0
    for t in range(steps):
        oracle.decoder_step(ring, w, F, np.arange(n), (pos0 + t).astype(np.int32), x)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"value": round(n * done / dt, 3), "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"{n} streams x {done} decode steps of the 12-layer decoder (oracle restatement of "
                      f"ref-decode.mjs decodeStep: numpy GEMMs, C attention mirror), {dt:.1f} s"}


# ------------------------------------------------------------------ the local 17-step head
def local_weights(h, ffn, codes, channels, seed=0):
    """N(0, 0.02) weights in mb_local_head_create's order, LayerNorm gains 1,
    N(0,1) embedding rows, text-head columns N(0, 1/h)."""
    from mockbird_b200.engine import LocalHead

    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(LocalHead.weight_count(h, ffn, codes, channels)) * 0.02).astype(np.float32)
    per = 2 * h + h * 3 * h + 3 * h + h * h + h + 2 * h + h * ffn + ffn + ffn * h + h
    w[0:h] = 1.0
    w[2 * h + 3 * h * h + 3 * h + h * h + h: 2 * h + 3 * h * h + 3 * h + h * h + 2 * h] = 1.0
    w[per:per + h] = 1.0
    off = per + 2 * h
    w[off:off + h] = rng.standard_normal(h)
    w[off + h:off + 3 * h] = rng.standard_normal(2 * h) / np.sqrt(h)
    off += 3 * h
    m = (channels - 1) * codes * h
    w[off:off + m] = rng.standard_normal(m)
    return w


def local_algo(n, h, ffn, codes, channels):
    """Algorithmic FLOPs and bytes of one frame for n streams: the layer's four
    GEMMs at every step, the audio-head GEMM at every step but the first; bytes =
    the bf16 weights each step reads + the embedding rows + hidden in / tokens out."""
    steps = channels + 1
    layer_params = 4 * h * h + 2 * h * ffn
    head_params = h * codes
    flops = 2.0 * n * (steps * layer_params + channels * head_params)
    weight_bytes = 2.0 * (steps * layer_params + channels * head_params)
    act_bytes = 4.0 * n * ((channels - 1) * h + h + channels + 1)
    return flops, weight_bytes + act_bytes


def run_local(args, cfg, rank, world, device):
    import torch

    from mockbird_b200 import KvRing, LocalHead
    from mockbird_b200.scheduler import max_over_ranks

    n, F, codes, ch = cfg["streams"], cfg["ffn"], cfg["codes"], cfg["channels"]
    ring = KvRing(layers=1, capacity=ch + 1, streams=n, dtype=cfg["dtype"], wrap=False, max_position=ch + 1,
                  device=device.index)
    head = LocalHead(ring, local_weights(HID, F, codes, ch), F, codes, ch, 1.2)
    g = torch.Generator(device=device)
    g.manual_seed(91 + rank)
    hidden = torch.randn(8, n, HID, generator=g, device=device)  # global hidden states, rotating
    streams = torch.arange(n, dtype=torch.int32, device=device)
    K, W = args.steps, args.warmup
    for t in range(W):
        head.frame(streams, hidden[t % 8])
    ring.sync()
    dist = _dist()
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device.index)
    clocks.start()
    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for t in range(W, W + K):
        tok, cont, _ = head.frame(streams, hidden[t % 8])
    ev1.record(stream)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ring.sync()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, device if dist else None)
    # e2e: the hidden states from pinned host memory in, tokens and the stop flags out, every frame
    host_in = torch.empty(2, n, HID).pin_memory()
    host_in.copy_(hidden[:2].cpu())
    host_tok = torch.empty(n, ch, dtype=torch.int32).pin_memory()
    host_cont = torch.empty(n, dtype=torch.int32).pin_memory()
    ids = np.arange(n, dtype=np.int32)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for t in range(K):
        head.frame_host(ids, host_in[t % 2], host_tok, host_cont)
    e2e_s = max_over_ranks(time.perf_counter() - t0, device if dist else None)
    flops, byts = local_algo(n, HID, F, codes, ch)
    tpeak, tkind = tensor_peak()
    hpeak, hkind = peaks()
    t_s = ms / 1e3 / K
    value = world * n * K / (ms_max / 1e3)
    graph = os.environ.get("MOCKBIRD_LOCAL_GRAPH", "1") != "0"
    result = {
        "metric": LOCAL_METRIC, "value": round(value, 1), "unit": "frames/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms_max / K, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (seeded N(0,1) hidden states, N(0,0.02) weights)",
        "config": {"workload": cfg["workload"], "streams_per_gpu": n, "global_streams": n * world,
                   "ffn": F, "codes": codes, "channels": ch,
                   "parallelism": f"stream-sharded x{world} (no collective)",
                   "l2": "weights (15.7 MB per step) are re-read every step and may stay in L2; the bound is "
                         "the tensor pipe at this batch", "cuda_graph": graph,
                   "value_per_gpu": round(value / world, 1),
                   "gemms": "this library's tcgen05 GEMMs; embedding, LayerNorm, attention, text-head decision "
                            "and argmax are this library's kernels too"},
        "roofline": {"bound": "tensor", "achieved": round(flops / t_s / 1e12, 2), "peak": tpeak,
                     "unit": "TFLOP/s", "frac": round(flops / t_s / 1e12 / tpeak, 4), "traffic": None,
                     "peak_source": f"{tkind} bf16_tflops (burst)",
                     "hbm_achieved_gbs": round(byts / t_s / 1e9, 1), "hbm_peak": hpeak,
                     "timing": "CUDA events over the timed frames; algorithmic FLOPs = the layer's GEMMs at 17 "
                               "steps + the audio-head GEMMs at 16 steps"},
        "e2e": {"value": round(world * n * K / e2e_s, 1), "unit": "frames/s",
                "h2d_bytes_per_step": n * HID * 4, "d2h_bytes_per_step": n * (ch + 1) * 4,
                "api": "mb_local_head_frame_host (C ABI): the hidden states from pinned host memory in, the "
                       "tokens and stop flags back to pinned host memory, one synchronisation per frame"},
        "gpu_launches": K * ((ch + 1) * 9 + 1),
        "gpu_launches_note": "per step: LN2, ln_f, attention, the layer's 4 GEMMs, and the text decision (step 0) or "
                             "the audio-head GEMM and the argmax (steps 1-16, the argmax also embedding and applying "
                             "LN1 for the next step); steps 0 and 1 embed with their own kernel",
        "clocks": clk,
    }
    head.dispose()
    return result, ring


def run_cpu_local(cfg, frames, sample_streams=2, budget_s=None):
    """The reference's local head (ref-decode.mjs localStep/argmaxPenalty restated by the oracle) on the host."""
    use_all_host_threads()
    import oracle

    n, F, codes, ch = sample_streams, cfg["ffn"], cfg["codes"], cfg["channels"]
    ring = oracle.Ring(layers=1, streams=n, heads=H, capacity=ch + 1, dtype=cfg["dtype"], wrap=False,
                       max_position=ch + 1)
    w = local_weights(HID, F, codes, ch)
    seen = np.zeros((n, ch, codes // 32), np.uint32)
    x = np.random.default_rng(6).standard_normal((n, HID)).astype(np.float32)
    t0 = time.perf_counter()
    done = 0
    for _ in range(frames):
        oracle.local_frame(ring, w, F, codes, ch, 1.2, np.arange(n), x, seen)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"value": round(n * done / dt, 3), "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"{n} streams x {done} local-head frames (oracle restatement of ref-decode.mjs localStep + "
                      f"argmaxPenalty: numpy GEMMs, C attention mirror), {dt:.1f} s"}


# ------------------------------------------------------------------ CPU reference (oracle port)
def run_cpu(cfg, steps, warmup, sample_streams, budget_s=None):
    """The reference algorithm (oracle mirror of the WGSL kernels) on the host cores:
    `sample_streams` streams of the workload, all 12 layers per frame."""
    use_all_host_threads()
    import oracle

    n, L, C = sample_streams, cfg["layers"], cfg["capacity"]
    ring = oracle.Ring(layers=L, streams=n, heads=H, capacity=C, dtype=cfg["dtype"], wrap=True,
                       max_position=8192)
    rng = np.random.default_rng(7)
    if cfg["job_steps"] is None:
        lengths0 = config5_lengths(4096, C)[:n].astype(np.int64)
        kvv = ring.kv_view()
        for s, Ls in enumerate(lengths0):
            if Ls > 1:
                rows = rng.standard_normal((2, H, int(Ls) - 1, HD)).astype(np.float32)
                if cfg["dtype"] == "f32":
                    kvv[:, s, :, :, :Ls - 1] = rows[None]
                else:
                    u = rows.view(np.uint32)
                    kvv[:, s, :, :, :Ls - 1] = ((u >> 16).astype(np.uint16))[None]
                ring.slot_pos[:, s, :Ls - 1] = np.arange(Ls - 1)
    else:
        lengths0 = None
    qkv = rng.standard_normal((4, L, n, QKV)).astype(np.float32)
    ids = np.arange(n, dtype=np.int32)

    def frame(t):
        pos = positions_for(cfg, t, n, lengths0)
        for layer in range(L):
            ring.append_attend(layer, ids, pos, qkv[t % 4, layer])

    for t in range(warmup):
        frame(t)
    if lengths0 is None:
        ring.reset()
    t0 = time.perf_counter()
    done = 0
    for t in range(steps):
        if lengths0 is None and t > 0 and t % cfg["job_steps"] == 0:
            ring.reset()
        frame(t if lengths0 is None else warmup + t)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    if lengths0 is None:
        what = (f"the whole {cfg['job_steps']}-step job (positions 0..{cfg['job_steps'] - 1})"
                if done == cfg["job_steps"] else f"the first {done} steps of the job (time budget)")
    else:
        what = f"{done} consecutive steps from the seeded live lengths"
    return {"value": round(n * done / dt, 2), "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"{n} of the workload's streams x {what}, all {L} layers per frame, oracle/oracle.c fp32 "
                      f"mirror of the WGSL kernels, OpenMP over (stream, head), {dt:.1f} s"}


def cpu_job_steps(cfg, steps):
    """Steps of a CPU leg: config 2's whole job (its windows grow, then wrap, so
    a prefix would time only short windows); for config 5 its default 200
    serving steps, or more if the GPU arm runs more."""
    if cfg["job_steps"] is not None:
        return cfg["job_steps"]
    return max(steps, cfg["steps"])


def run_cpu_prefill(cfg, steps, warmup, sample_streams=1, budget_s=None):
    """The reference's prefill (ROPE_SPLIT_CACHE + ATTENTION_SCORES/_SOFTMAX/_APPLY,
    oracle restatement) on the host cores: `sample_streams` streams x 12 layers per step."""
    use_all_host_threads()
    import oracle

    n, L, C, S = sample_streams, cfg["layers"], cfg["capacity"], cfg["rows"]
    ring = oracle.Ring(layers=L, streams=n, heads=H, capacity=C, dtype=cfg["dtype"], wrap=True, max_position=4096)
    qkv = (np.random.default_rng(9).standard_normal((L, n, S, QKV)) * 0.5).astype(np.float32)
    ids = np.arange(n, dtype=np.int32)
    for _ in range(warmup):
        ring.prefill(0, ids, qkv[0], q_round=True)
    t0 = time.perf_counter()
    done = 0
    for _ in range(steps):
        for layer in range(L):
            ring.prefill(layer, ids, qkv[layer], q_round=True)
        done += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"value": round(prefill_flops(S, n, L) * done / dt / 1e12, 5), "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"{n} stream(s) x {done} step(s) of the 12-layer {S}-row prefill, oracle/oracle.c fp32 "
                      f"restatement of ROPE_SPLIT_CACHE + ATTENTION_*, OpenMP over (stream, head), {dt:.1f} s"}


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS),
                    help="1-5: BASELINE configs; 6: the local 17-step head")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--start", type=int, default=None,
                    help="config 2 profiling variant: begin at this position with full windows pre-written "
                         "(steady state, no resets) instead of the 1500-frame job")
    ap.add_argument("--streams", type=int, default=None, help="override streams per GPU (small profiling cases)")
    ap.add_argument("--ring-dtype", default=None, choices=["f32", "bf16", "f16"],
                    help="override the ring's storage type (e.g. config 3 on an fp32 ring)")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.streams:
        cfg["streams"] = args.streams
        cfg["workload"] += f" [profiling case: {args.streams} streams/GPU]"
    if args.ring_dtype and args.ring_dtype != cfg["dtype"]:
        cfg["workload"] += f" [ring storage {args.ring_dtype} instead of {cfg['dtype']}]"
        cfg["dtype"] = args.ring_dtype
    if args.start is not None:
        if cfg["job_steps"] is None or args.start < cfg["capacity"]:
            ap.error("--start applies to config 2 with a position >= capacity")
        cfg["start"] = args.start
        cfg["workload"] += f" [steady-state variant: positions from {args.start}, full windows]"
    args.steps = args.steps if args.steps is not None else cfg["steps"]
    args.warmup = args.warmup if args.warmup is not None else cfg["warmup"]
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.config == 1:
            base = run_cpu_single(cfg, args.steps, budget_s=120.0)
            metric, unit = METRIC, "frames/s"
        elif args.config == 3:
            base = run_cpu_prefill(cfg, args.steps, 1, sample_streams=1, budget_s=120.0)
            metric, unit = "causal prefill attention TFLOP/s (config 3; RoPE+cache write and attention, all 12 layers)", "TFLOP/s"
        elif args.config == 4:
            base = run_cpu_decoder(cfg, args.steps, sample_streams=2, budget_s=120.0)
            metric, unit = METRIC, "frames/s"
        elif args.config == 6:
            base = run_cpu_local(cfg, args.steps, sample_streams=2, budget_s=120.0)
            metric, unit = LOCAL_METRIC, "frames/s"
        else:
            base = run_cpu(cfg, cpu_job_steps(cfg, args.steps), args.warmup, sample_streams=4, budget_s=240.0)
            metric, unit = METRIC, "frames/s"
        line = {"metric": metric, "value": base["value"], "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic", "impl": "reference",
                "config": {"workload": cfg["workload"]},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": "reference = CPU restatement of the reference's WGSL kernels (oracle/); the WGSL itself needs "
                        "a WebGPU runtime and Node, unavailable on this box"}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from mockbird_b200.scheduler import init_group
        init_group("nccl", timeout_s=300, device=device)
    if args.config == 1:
        result, ring = run_single(args, cfg, rank, world, device)
    elif args.config == 3:
        result, ring = run_prefill(args, cfg, rank, world, device)
    elif args.config == 4:
        result, ring = run_decoder(args, cfg, rank, world, device)
    elif args.config == 6:
        result, ring = run_local(args, cfg, rank, world, device)
    else:
        result, ring = run_ours(args, cfg, rank, world, device)
    dist = _dist()
    if dist:
        from mockbird_b200.scheduler import gather_reports
        gather_reports({"rank": rank, "value_gpu": result["value"] / world}, device)
    if rank == 0 and world == 1 and not args.no_cpu and cfg.get("start") is None:
        if args.config == 1:
            result["cpu_baseline"] = run_cpu_single(cfg, args.steps, budget_s=20.0)
        elif args.config == 3:
            result["cpu_baseline"] = run_cpu_prefill(cfg, 1, 0, sample_streams=1, budget_s=30.0)
        elif args.config == 4:
            result["cpu_baseline"] = run_cpu_decoder(cfg, 3, sample_streams=2, budget_s=30.0)
        elif args.config == 6:
            result["cpu_baseline"] = run_cpu_local(cfg, 3, sample_streams=2, budget_s=30.0)
        else:
            result["cpu_baseline"] = run_cpu(cfg, cpu_job_steps(cfg, args.steps), 2, sample_streams=4,
                                             budget_s=60.0)
    elif rank == 0:
        result["cpu_baseline"] = None
    ring.dispose()
    if rank == 0:
        print(json.dumps(result), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
