#!/usr/bin/env python
"""Benchmark of the int8 NHWC conv hot path on B200 (one JSON line on rank 0).

Workload (the large pointwise pair, int8 end to end): per GPU a batch of 512
NHWC images at 14x14:  y1 = conv1x1(x, C=1024 -> K=2048),  y2 = conv1x1(y1, C=2048 -> K=512),
both with int32 bias + per-channel fp32 scale + round-half-even + clamp to int8 (fused epilogue).
One step = both layers over the batch.  Inputs / weights: seeded synthetic int8 U[-127,127],
bias U[-2^15,2^15], scales U[1e-4,1e-3], generated on the device by the library's counter-based
generator (random-init weights; no dataset exists for this benchmark).

Multi-GPU (torchrun, one process per GPU): every rank runs its own batch of 512 images (weak
scaling, weights replicated, no collective on the data path); the timed region is bracketed by a
barrier + synchronize, and the time is the max over ranks.  NCCL gathers only output checksums
after timing (verification).

`--impl reference` times the reference's own CPU implementation of the path
(src/cpu_ref.cpp cpu_fprop_nhwc_qi32, compiled from the reference sources into
oracle/_ref/libref_oracle.so, threaded over images) on a bounded sample of the same workload,
followed by the requantization epilogue of the CPU oracle.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int8 conv TOPS/GPU (% of dense int8 peak) and images/sec at 1/2/4/8 B200"
BATCH, HW = 512, 14
LAYERS = [(1024, 2048), (2048, 512)]  # (C, K) of the two 1x1 convs
SEED = 42


def ops_per_image() -> int:
    return sum(2 * HW * HW * c * k for c, k in LAYERS)


def bytes_per_image() -> int:
    # algorithmic HBM bytes: int8 input + int8 output per layer (weights, bias, scales are per launch)
    return sum(HW * HW * (c + k) for c, k in LAYERS)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            keep = {v.strip() for v in vis.split(",")}
            rows = [r for r in rows if r[0].strip() in keep] or rows
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 600] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------- our arm

def headline_config(world: int) -> dict:
    """`config` of the headline line; both arms print exactly this dict."""
    return {"workload": "config4 pointwise 1x1 pair: b512 14x14 C1024->K2048 then C2048->K512, "
                        "bias+per-channel requant int8 epilogue",
            "global_batch": BATCH * world, "per_gpu_batch": BATCH, "parallelism": f"dp{world} (batch shards)",
            "l2": "flushed between timed steps (256 MiB write outside the events)"}


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import synth, _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    (c1, k1), (c2, k2) = LAYERS
    # per-rank shard of the synthetic batch: images [rank*512, rank*512+512) of one global stream
    x = torch.empty((BATCH, HW, HW, c1), dtype=torch.int8, device=dev)
    # tensor ids: 1 input, 2/3 weights, 4/5 bias, 6/7 scales; rank offset in the seed stream
    synth.fill_s8_uniform(x, SEED + rank, 1)
    w1 = synth.fill_s8_uniform(torch.empty((k1, 1, 1, c1), dtype=torch.int8, device=dev), SEED, 2)
    w2 = synth.fill_s8_uniform(torch.empty((k2, 1, 1, c2), dtype=torch.int8, device=dev), SEED, 3)
    b1 = synth.fill_i32_uniform(torch.empty(k1, dtype=torch.int32, device=dev), SEED, 4, -2**15, 2**15)
    b2 = synth.fill_i32_uniform(torch.empty(k2, dtype=torch.int32, device=dev), SEED, 5, -2**15, 2**15)
    s1 = torch.from_numpy(synth.scales_f32(k1, SEED, 6)).to(dev)
    s2 = torch.from_numpy(synth.scales_f32(k2, SEED, 7)).to(dev)
    y1 = torch.empty((BATCH, HW, HW, k1), dtype=torch.int8, device=dev)
    y2 = torch.empty((BATCH, HW, HW, k2), dtype=torch.int8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)  # > 126 MB L2
    p = b2q.Conv2DParams(0, 0, 1, 1, 1, 1, 1)
    epi = b2q.Epilogue.int8()

    def step(xin):
        b2q.conv2d_s8_into(y1, xin, w1, b1, s1, BATCH, HW, HW, c1, 1, 1, k1, p, epi)
        b2q.conv2d_s8_into(y2, y1, w2, b2, s2, BATCH, HW, HW, c2, 1, 1, k2, p, epi)

    for _ in range(args.warmup):
        step(x)
    assert b2q.last_path().startswith("tcgen05-tiled"), b2q.last_path()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-timed region: K steps, L2 flushed between steps (outside the events)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
    launches0 = b2q.tc_launch_count()
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(i & 0x7F)
        e0, e1, e2 = ev[i]
        e0.record(stream)
        b2q.conv2d_s8_into(y1, x, w1, b1, s1, BATCH, HW, HW, c1, 1, 1, k1, p, epi)
        e1.record(stream)
        b2q.conv2d_s8_into(y2, y1, w2, b2, s2, BATCH, HW, HW, c2, 1, 1, k2, p, epi)
        e2.record(stream)
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - wall0
    clocks = sampler.stop() if rank == 0 else None
    launches = b2q.tc_launch_count() - launches0
    t1 = [a.elapsed_time(b) for a, b, _ in ev]
    t2 = [b.elapsed_time(c) for _, b, c in ev]
    sustained = sustained_window(step, x, flush, stream, barrier, rank, args.sustain_s)
    step_ms = sum(t1) / len(t1) + sum(t2) / len(t2)
    total_ms = sum(t1) + sum(t2)
    if _lib.lib().b200q_device_error() != 0:
        raise RuntimeError(_lib.lib().b200q_last_error().decode())

    # ---- end to end through the public API: pinned host input -> device -> both layers -> host
    # output, with the batch cut into chunks so H2D, kernels and D2H overlap (ConvStack.run_host)
    from my_own_cnn_b200.stack import ConvLayer, ConvStack

    net = ConvStack([ConvLayer(w1, b1, s1, p, epi), ConvLayer(w2, b2, s2, p, epi)], (HW, HW, c1))
    xh = torch.empty_like(x, device="cpu").pin_memory()
    xh.copy_(x.cpu())
    yh = torch.empty_like(y2, device="cpu").pin_memory()
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        net.run_host(xh, yh, chunk=args.chunk)
    torch.cuda.synchronize()
    barrier()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(stream)
    for _ in range(e2e_steps):
        net.run_host(xh, yh, chunk=args.chunk)
    e_ev.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = s_ev.elapsed_time(e_ev) / e2e_steps
    if not torch.equal(yh, y2.cpu()):
        raise RuntimeError("pipelined host pass differs from the device-resident pass")

    # ---- after timing: max over ranks of the device times, and a checksum gather (verification)
    from my_own_cnn_b200.shard import checksum, gather_tensors, max_over_ranks

    total_ms, e2e_ms = max_over_ranks([total_ms, e2e_ms], device=dev)
    step_ms = total_ms / args.steps
    chk = torch.cat([checksum(y2), checksum(y1)])
    checksums = [g.tolist() for g in gather_tensors(chk)]
    strong = strong_scaling(args, x, w1, w2, b1, b2, s1, s2, y1, y2, flush, stream, barrier, rank, world) \
        if world > 1 else None
    if rank != 0:
        return None

    peaks = load_peaks()
    int8_peak_tops = 2.0 * peaks["bf16_tflops"]  # dense int8 = 2x dense bf16 on B200
    ops_step = ops_per_image() * BATCH
    img_per_s = world * BATCH / (step_ms * 1e-3)
    tops_per_gpu = ops_step / (step_ms * 1e-3) / 1e12
    # roofline of the dominant kernel (tc_gemm_s8_kernel, both launches): algorithmic ops per
    # launch / mean CUDA-event launch time
    mean1, mean2 = sum(t1) / len(t1), sum(t2) / len(t2)
    achieved = ops_step / ((mean1 + mean2) * 1e-3) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "tc_gemm_s8_pointwise_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("bytes_per_step")
    h2d = x.numel()
    d2h = y2.numel()
    out = {
        "metric": METRIC,
        "value": round(img_per_s, 1),
        "unit": "images/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "s8xs8->s32",
        "data": "synthetic (seeded splitmix64, random-init int8 weights)",
        "config": headline_config(world),
        "tops_per_gpu": round(tops_per_gpu, 1),
        "frac_of_int8_peak": round(tops_per_gpu / int8_peak_tops, 4),
        "layer_ms": [round(mean1, 5), round(mean2, 5)],
        "e2e": {"value": round(world * BATCH / (e2e_ms * 1e-3), 1), "unit": "images/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": f"my_own_cnn_b200.stack.ConvStack.run_host (C ABI b200q_conv2d_s8), pinned host buffers, {args.chunk}-image chunks, H2D/compute/D2H overlapped"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(int8_peak_tops, 1),
                     "unit": "TOP/s", "frac": round(achieved / int8_peak_tops, 4), "traffic": traffic,
                     "kernel": "tc_gemm_s8_kernel (layer 1) + tc_gemm_s8_pair_kernel (layer 2)",
                     "peak_source": f"2 x bf16_tflops ({peaks['source']}) = dense int8 peak"},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "wall_s_timed": round(wall, 3),
        "sustained": sustained,
        **({"strong": strong} if strong else {}),
        "verify": {"checksums_y2_y1_per_rank": checksums},
    }
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    return out


def strong_scaling(args, x, w1, w2, b1, b2, s1, s2, y1, y2, flush, stream, barrier, rank: int, world: int) -> dict:
    """Strong scaling of the headline: one global batch of 512 images split over the ranks
    (shard_range: contiguous, balanced), the same two layers, max over ranks of the device time."""
    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200.shard import max_over_ranks, shard_range

    (c1, k1), (c2, k2) = LAYERS
    start, cnt = shard_range(BATCH, rank, world)
    p = b2q.Conv2DParams(0, 0, 1, 1, 1, 1, 1)
    epi = b2q.Epilogue.int8()
    xs, y1s, y2s = x[:cnt], y1[:cnt], y2[:cnt]

    def step():
        b2q.conv2d_s8_into(y1s, xs, w1, b1, s1, cnt, HW, HW, c1, 1, 1, k1, p, epi)
        b2q.conv2d_s8_into(y2s, y1s, w2, b2, s2, cnt, HW, HW, c2, 1, 1, k2, p, epi)

    for _ in range(args.warmup):
        step()
    paths = b2q.last_path()
    barrier()
    torch.cuda.synchronize()
    ms = _timed_ms(step, args.steps, flush, stream)
    barrier()
    (total,) = max_over_ranks([sum(ms)], device=x.device)
    step_ms = total / args.steps
    return {"scaling": "strong", "global_batch": BATCH, "per_gpu_batch": f"{BATCH // world}-{-(-BATCH // world)}",
            "value": round(BATCH / (step_ms * 1e-3), 1), "unit": "images/s", "ms_per_step": round(step_ms, 5),
            "layer2_path_rank0": paths}


def sustained_window(step, x, flush, stream, barrier, rank: int, seconds: float) -> dict | None:
    """The headline step back to back for at least `seconds` (L2 flushed between steps, outside the
    events), with the clocks sampled over the whole window: a long enough record to show the clocks
    the headline's short timed region ran at."""
    import torch

    if seconds <= 0:
        return None
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
    barrier()
    torch.cuda.synchronize()
    n, dev_ms, t0 = 0, 0.0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        evs = []
        for i in range(50):
            flush.fill_(i & 0x7F)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step(x)
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        dev_ms += sum(a.elapsed_time(b) for a, b in evs)
        n += len(evs)
    barrier()
    clocks = sampler.stop() if rank == 0 else None
    from my_own_cnn_b200.shard import max_over_ranks

    (dev_ms,) = max_over_ranks([dev_ms], device=x.device)
    return {"steps": n, "device_s": round(dev_ms / 1e3, 3), "wall_s": round(time.perf_counter() - t0, 2),
            "ms_per_step": round(dev_ms / n, 5), "images_per_s_per_gpu": round(BATCH / (dev_ms / n * 1e-3), 1),
            "clocks": clocks}


# ---------------------------------------------------------------------- CPU baseline

def _cpu_sample(images: int, threads: int):
    """Reference cpu_fprop_nhwc_qi32 (+ oracle requant) on `images` images of both layers."""
    import numpy as np

    from my_own_cnn_b200 import synth
    from oracle import oracle

    (c1, k1), (c2, k2) = LAYERS
    x = synth.s8_uniform_host(SEED, 1, -127, 127, 0, images * HW * HW * c1).astype(np.float32)
    w1 = synth.s8_uniform_host(SEED, 2, -127, 127, 0, k1 * c1).astype(np.float32)
    w2 = synth.s8_uniform_host(SEED, 3, -127, 127, 0, k2 * c2).astype(np.float32)
    b1 = synth.i32_uniform_host(SEED, 4, -2**15, 2**15, 0, k1)
    b2 = synth.i32_uniform_host(SEED, 5, -2**15, 2**15, 0, k2)
    s1, s2 = synth.scales_f32(k1, SEED, 6), synth.scales_f32(k2, SEED, 7)
    use_ref = oracle.ref_available()
    a1 = oracle.conv_args(images, HW, HW, c1, 1, 1, k1, 0, 0)
    a2 = oracle.conv_args(images, HW, HW, c2, 1, 1, k2, 0, 0)

    def run():
        if use_ref:
            acc1 = oracle.ref_conv_qi32_threaded(a1, x, w1, threads)
            y1 = oracle.requant_s8(acc1, b1, s1)
            acc2 = oracle.ref_conv_qi32_threaded(a2, y1.astype(np.float32), w2, threads)
        else:
            acc1 = oracle.conv_s8(a1, x.astype(np.int8), w1.astype(np.int8), threads)
            y1 = oracle.requant_s8(acc1, b1, s1)
            acc2 = oracle.conv_s8(a2, y1, w2.astype(np.int8), threads)
        return oracle.requant_s8(acc2, b2, s2)

    return run, ("reference" if use_ref else "port")


def cpu_baseline(budget_s: float) -> dict:
    from oracle import oracle

    threads = oracle.cpu_threads()
    images = max(1, threads)
    run, kind = _cpu_sample(1, threads)
    t0 = time.perf_counter()
    run()
    t_one = time.perf_counter() - t0  # one image, one thread busy
    images = int(max(threads, min(512, budget_s / max(t_one, 1e-3) * threads * 0.8)))
    images = max(threads, (images // threads) * threads)
    run, kind = _cpu_sample(images, threads)
    t0 = time.perf_counter()
    run()
    dt = time.perf_counter() - t0
    return {"value": round(images / dt, 3), "unit": "images/s", "cores": threads, "kind": kind,
            "sample": f"{images} images of the same two-layer workload (of {BATCH}), images split over "
                      f"{threads} threads; src/cpu_ref.cpp cpu_fprop_nhwc_qi32 on float codes + CPU requant",
            "seconds": round(dt, 2), "tops": round(images * ops_per_image() / dt / 1e12, 5)}


def run_reference(args) -> dict:
    from oracle import oracle

    threads = oracle.cpu_threads()
    run, kind = _cpu_sample(threads, threads)
    t0 = time.perf_counter()
    run()
    t_probe = time.perf_counter() - t0
    # size each step at ~budget seconds of work, at least one image per thread
    per_step_budget = max(1.0, min(20.0, args.cpu_seconds))
    images = max(threads, int(per_step_budget / max(t_probe, 1e-3)) * threads)
    images = min(images, BATCH)
    run, kind = _cpu_sample(images, threads)
    for _ in range(max(0, min(args.warmup, 1))):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    ms = statistics.mean(times) * 1e3
    val = images / (ms * 1e-3)
    return {
        "metric": METRIC, "value": round(val, 3), "unit": "images/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "s8xs8->s32", "data": "synthetic (seeded splitmix64)",
        "config": headline_config(args.gpus),
        "impl": "reference",
        "cpu_baseline": {"value": round(val, 3), "unit": "images/s", "cores": threads, "kind": kind,
                         "sample": f"{images} of the {BATCH} images of the workload per step, images split over "
                                   f"{threads} threads; src/cpu_ref.cpp cpu_fprop_nhwc_qi32 + CPU requant"},
        "e2e": {"value": round(val, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference_gpu(args) -> list[dict]:
    """Secondary baseline: the reference's own CUDA quantized conv (src/cuda_kernels.cu:1336-1392:
    per-call cudaMalloc/cudaFree, im2col to int32, SIMT int32 GEMM, unpack; compiled unmodified into
    oracle/_ref/libref_gpu.so) against this library's drop-in for the same entry point
    (launch_fprop_nhwc_qi32, float codes, S5 zero points 0) and its int8 entry, on BASELINE
    configs 1 and 4.  One JSON record per case, with an identical-int32 check."""
    import ctypes

    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import synth

    lib = ROOT / "oracle" / "_ref" / "libref_gpu.so"
    if not lib.exists():
        return [{"impl": "reference-gpu", "unavailable": "oracle/_ref/libref_gpu.so was not built"}]
    ref = ctypes.CDLL(str(lib))
    ref.refgpu_fprop_qi32_s5.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 9 + [ctypes.c_void_p] * 2
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    cases = [("config1 3x3 N1 56x56 C64->K64", 1, 56, 56, 64, 3, 64, 1, 1),
             ("config4a 1x1 b512 14x14 C1024->K2048", 512, 14, 14, 1024, 1, 2048, 0, 1),
             ("config4b 1x1 b512 14x14 C2048->K512", 512, 14, 14, 2048, 1, 512, 0, 1)]
    out = []
    for name, n, h, w, c, r, k, pad, st in cases:
        x8 = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device=dev), SEED, 1)
        w8 = synth.fill_s8_uniform(torch.empty((k, r, r, c), dtype=torch.int8, device=dev), SEED, 2)
        xf, wf = x8.float(), w8.float()
        p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, 1)
        ho, wo = b2q.conv_out_shape(h, w, c, r, r, k, p)
        y_ref = torch.empty((n, ho, wo, k), dtype=torch.int32, device=dev)
        y_drop = torch.empty_like(y_ref)
        y_s8 = torch.empty_like(y_ref)
        qp_in = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)] * n)
        qp_f = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)])

        def run_ref():
            assert ref.refgpu_fprop_qi32_s5(xf.data_ptr(), wf.data_ptr(), y_ref.data_ptr(), n, h, w, c, r, r, k, pad,
                                            st, qp_in.data_ptr(), qp_f.data_ptr()) == 0

        run_drop = lambda: b2q.launch_fprop_nhwc_qi32(xf, wf, y_drop, n, h, w, c, r, r, k, p, qp_in, qp_f,
                                                      qtype=b2q.DataType.LinQuantS5)
        run_s8 = lambda: b2q.conv2d_s8_into(y_s8, x8, w8, None, None, n, h, w, c, r, r, k, p, b2q.Epilogue.int32())
        run_ref(); run_drop(); drop_path = b2q.last_path(); run_s8(); s8_path = b2q.last_path()
        t_ref = statistics.median(_timed_ms(run_ref, 3, flush, stream))
        t_drop = statistics.median(_timed_ms(run_drop, 20, flush, stream))
        t_s8 = statistics.median(_timed_ms(run_s8, 20, flush, stream))
        ops = 2 * n * ho * wo * k * r * r * c
        out.append({"impl": "reference-gpu", "case": name, "reference_gpu_ms": round(t_ref, 4),
                    "dropin_qi32_ms": round(t_drop, 4), "dropin_path": drop_path,
                    "int8_entry_ms": round(t_s8, 4), "int8_entry_path": s8_path,
                    "dropin_speedup": round(t_ref / t_drop, 1), "int8_speedup": round(t_ref / t_s8, 1),
                    "dropin_tops": round(ops / t_drop / 1e9, 1),
                    "identical_int32": bool(torch.equal(y_ref, y_drop) and torch.equal(y_ref, y_s8))})
        del xf, wf, y_ref, y_drop, y_s8
        torch.cuda.empty_cache()
    out += _reference_gpu_f32(ref, dev, stream, flush)
    return out


def _reference_gpu_f32(ref, dev, stream, flush) -> list[dict]:
    """The reference's fp32 conv (fprop / bprop / grad) and fp32 bmm against this library's fp32
    drop-ins on the same inputs: resnet_like_56x56 of the reference's conv_bench suite
    (src/main.cpp:163-186) and BASELINE config 2's bmm shape in fp32.  Agreement is reported as the
    largest |ours - reference| relative to the largest |reference|."""
    import ctypes

    import torch

    import my_own_cnn_b200 as b2q

    if not hasattr(ref, "refgpu_conv_f32"):
        return []
    ref.refgpu_conv_f32.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 10
    ref.refgpu_bmm_f32.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 6
    out = []
    n, h, w, c, k, r = 32, 56, 56, 64, 64, 3
    p = b2q.Conv2DParams(1, 1, 1, 1, 1, 1, 1)
    g = torch.Generator(device=dev).manual_seed(SEED)
    x = torch.randn((n, h, w, c), device=dev, generator=g)
    wt = torch.randn((k, r, r, c), device=dev, generator=g)
    dy = torch.randn((n, h, w, k), device=dev, generator=g)
    flops = 2.0 * n * h * w * k * r * r * c
    for op, name, a, b, shape, ours in (
            (0, "fprop", x, wt, (n, h, w, k), b2q.launch_fprop_nhwc),
            (1, "bprop", dy, wt, (n, h, w, c), b2q.launch_bprop_nhwc),
            (2, "grad", x, dy, (k, r, r, c), b2q.launch_grad_nhwc)):
        y_ref = torch.empty(shape, device=dev)
        y_me = torch.empty(shape, device=dev)
        run_ref = lambda: ref.refgpu_conv_f32(op, a.data_ptr(), b.data_ptr(), y_ref.data_ptr(), n, h, w, c, r, r, k, 1,
                                              1, 1)
        run_me = lambda: ours(a, b, y_me, n, h, w, c, r, r, k, p)
        run_ref(); run_me(); path = b2q.last_path()
        t_ref = statistics.median(_timed_ms(run_ref, 3, flush, stream))
        t_me = statistics.median(_timed_ms(run_me, 10, flush, stream))
        rel = float((y_me - y_ref).abs().max() / y_ref.abs().max())
        out.append({"impl": "reference-gpu", "case": f"fp32 {name} conv_bench resnet_like_56x56 (n32 56x56 C64 K64 3x3)",
                    "reference_gpu_ms": round(t_ref, 4), "ours_ms": round(t_me, 4), "ours_path": path,
                    "speedup": round(t_ref / t_me, 1), "ours_tflops": round(flops / t_me / 1e9, 1),
                    "max_rel_diff": rel})
    batch, M = 64, 1024
    A = torch.randn((batch, M, M), device=dev, generator=g)
    B = torch.randn((batch, M, M), device=dev, generator=g)
    C_ref, C_me = torch.empty_like(A), torch.empty_like(A)
    run_ref = lambda: ref.refgpu_bmm_f32(A.data_ptr(), B.data_ptr(), C_ref.data_ptr(), batch, M, M, M, 0, 0)
    run_me = lambda: b2q.bmm_matmul(A, B, C_me, batch, M, M, M, 0, 0)
    run_ref(); run_me(); path = b2q.last_path()
    t_ref = statistics.median(_timed_ms(run_ref, 3, flush, stream))
    t_me = statistics.median(_timed_ms(run_me, 10, flush, stream))
    out.append({"impl": "reference-gpu", "case": "fp32 bmm_matmul batch 64 x 1024^3 NN", "reference_gpu_ms": round(t_ref, 4),
                "ours_ms": round(t_me, 4), "ours_path": path, "speedup": round(t_ref / t_me, 1),
                "ours_tflops": round(2.0 * batch * M ** 3 / t_me / 1e9, 1),
                "max_rel_diff": float((C_me - C_ref).abs().max() / C_ref.abs().max())})
    # int32 bmm (bmm_matmul_i32) on config 2's shape with int8-range values held in int32
    if hasattr(ref, "refgpu_bmm_i32"):
        ref.refgpu_bmm_i32.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 6
        del A, B, C_ref, C_me
        Ai = torch.randint(-127, 128, (batch, M, M), dtype=torch.int32, device=dev, generator=g)
        Bi = torch.randint(-127, 128, (batch, M, M), dtype=torch.int32, device=dev, generator=g)
        Ci_ref, Ci_me = torch.empty_like(Ai), torch.empty_like(Ai)
        run_ref = lambda: ref.refgpu_bmm_i32(Ai.data_ptr(), Bi.data_ptr(), Ci_ref.data_ptr(), batch, M, M, M, 0, 0)
        run_me = lambda: b2q.bmm_matmul_i32(Ai, Bi, Ci_me, batch, M, M, M, 0, 0)
        run_ref(); run_me(); path = b2q.last_path()
        t_ref = statistics.median(_timed_ms(run_ref, 3, flush, stream))
        t_me = statistics.median(_timed_ms(run_me, 10, flush, stream))
        out.append({"impl": "reference-gpu", "case": "int32 bmm_matmul_i32 batch 64 x 1024^3 NN (int8-range values)",
                    "reference_gpu_ms": round(t_ref, 4), "ours_ms": round(t_me, 4), "ours_path": path,
                    "speedup": round(t_ref / t_me, 1), "identical": bool(torch.equal(Ci_me, Ci_ref))})
    return out


# ------------------------------------------------------------------ other BASELINE configs

NET_BATCH = {"resnet50": 256, "mobilenetv2": 512}


def run_net(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Configs 3 / 5: every conv of the network once per step over the per-GPU batch, each layer on
    its own resident synthetic input (max-pool and residual adds are not part of the conv path)."""
    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import _lib, nets
    from my_own_cnn_b200.shard import checksum, gather_tensors, max_over_ranks

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    specs = nets.NETS[args.config]()
    if args.layers:
        specs = [sp for sp in specs if re.fullmatch(args.layers, sp.name)]
        if not specs:
            raise SystemExit(f"--layers {args.layers!r} matches no layer of {args.config}")
    batch = args.batch or NET_BATCH[args.config]
    data = nets.NetData(specs, batch, SEED, dev, image_offset=rank)
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    for _ in range(args.warmup):
        data.run()
    paths = []
    for i in range(len(specs)):
        data.run_layer(i)
        paths.append(b2q.last_path())
    torch.cuda.synchronize()
    n = len(specs)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(n + 1)] for _ in range(args.steps)]
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
    launches0 = b2q.tc_launch_count()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for st in range(args.steps):
        flush.fill_(st & 0x7F)
        evs[st][0].record(stream)
        for i in range(n):
            data.run_layer(i)
            evs[st][i + 1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop() if rank == 0 else None
    launches = b2q.tc_launch_count() - launches0
    if _lib.lib().b200q_device_error() != 0:
        raise RuntimeError(_lib.lib().b200q_last_error().decode())
    layer_ms = [sum(evs[st][i].elapsed_time(evs[st][i + 1]) for st in range(args.steps)) / args.steps
                for i in range(n)]
    step_ms = sum(layer_ms)
    (step_ms,) = max_over_ranks([step_ms], device=dev)
    chk = torch.cat([checksum(data.layers[-1][5]), checksum(data.layers[0][5])])
    checksums = [g.tolist() for g in gather_tensors(chk)]
    if rank != 0:
        return None
    peaks = load_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    ops = [sp.ops_per_image() * batch for sp in specs]
    by_path = {}
    for sp, pth, ms, o in zip(specs, paths, layer_ms, ops):
        d = by_path.setdefault(pth, {"layers": 0, "ms": 0.0, "gop": 0.0, "bytes": 0})
        ho, wo = sp.out_hw()
        d["layers"] += 1
        d["ms"] += ms
        d["gop"] += o / 1e9
        d["bytes"] += batch * (sp.h * sp.w * sp.c + ho * wo * sp.k) + sp.k * sp.r * sp.r * (sp.c // sp.groups)
    for d in by_path.values():
        d["share"] = round(d["ms"] / step_ms, 4)
        d["tops"] = round(d["gop"] / d["ms"], 1) if d["ms"] else None
        d["gbs"] = round(d["bytes"] / d["ms"] / 1e6, 1) if d["ms"] else None
        d["ms"] = round(d["ms"], 4)
        d["gop"] = round(d["gop"], 2)
    tc = [v for k, v in by_path.items() if k.startswith("tcgen05")]
    tc_ms = sum(v["ms"] for v in tc)
    tc_tops = sum(v["gop"] for v in tc) / tc_ms if tc_ms else 0.0
    out = {
        "metric": METRIC, "value": round(world * batch / (step_ms * 1e-3), 1), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "s8xs8->s32",
        "data": "synthetic (seeded splitmix64; half-normal / normal int8 codes via quantile tables)",
        "config": {"workload": f"{args.config} conv stack, per-GPU batch {batch}, every conv on fresh input"
                   + (f", layers matching {args.layers!r} only" if args.layers else ""),
                   "global_batch": batch * world, "per_gpu_batch": batch, "parallelism": f"dp{world} (batch shards)",
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
        "tops_per_gpu": round(sum(ops) / (step_ms * 1e-3) / 1e12, 1),
        "frac_of_int8_peak": round(sum(ops) / (step_ms * 1e-3) / 1e12 / int8_peak, 4),
        "by_path": by_path,
        "roofline": {"bound": "tensor", "achieved": round(tc_tops, 1), "peak": round(int8_peak, 1), "unit": "TOP/s",
                     "frac": round(tc_tops / int8_peak, 4), "traffic": None, "kernel": "tc_gemm_s8_kernel (all layers)",
                     "peak_source": f"2 x bf16_tflops ({peaks['source']})"},
        "gpu_launches": int(launches), "clocks": clocks,
        "slowest_layers": sorted(({"layer": sp.name, "path": pth, "ms": round(ms, 4),
                                   "tops": round(o / ms / 1e9, 1)} for sp, pth, ms, o in zip(specs, paths, layer_ms, ops)),
                                 key=lambda d: -d["ms"])[:6],
        "verify": {"checksums_last_first_per_rank": checksums},
    }
    if "cuda-core-depthwise" in by_path:
        d = by_path["cuda-core-depthwise"]
        out["roofline_depthwise"] = {"bound": "hbm", "achieved": d["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                     "frac": round(d["gbs"] / peaks["hbm_gbs"], 4)}
    return out


def run_chain(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Configs 3 / 5 as chained networks: one step = the whole int8 forward of the per-GPU batch
    (stem, max pool, every conv fed by the previous layer, residual adds fused into the conv
    epilogues, global average pool), input resident in HBM."""
    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import _lib, nets, synth
    from my_own_cnn_b200.shard import checksum, gather_tensors, max_over_ranks

    net = args.config.replace("-chain", "")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    batch = args.batch or NET_BATCH[net]
    model = nets.ChainedNet(net, SEED, dev)
    x = torch.empty((batch, 224, 224, 3), dtype=torch.int8, device=dev)
    act = torch.from_numpy(nets.act_table()).to(dev)
    synth.fill_s8_table(x, SEED + rank, 1, act)  # each rank its own seeded images
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    for _ in range(args.warmup):
        y = model.forward(x)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler()
    if rank == 0:
        sampler.start()
    launches0 = b2q.tc_launch_count()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for st in range(args.steps):
        flush.fill_(st & 0x7F)
        evs[st][0].record(stream)
        y = model.forward(x)
        evs[st][1].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop() if rank == 0 else None
    launches = b2q.tc_launch_count() - launches0
    if _lib.lib().b200q_device_error() != 0:
        raise RuntimeError(_lib.lib().b200q_last_error().decode())
    step_ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    (step_ms,) = max_over_ranks([step_ms], device=dev)
    checksums = [g.tolist() for g in gather_tensors(checksum(y))]
    if rank != 0:
        return None
    peaks = load_peaks()
    ops = sum(sp.ops_per_image() for sp in model.specs) * batch
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = chain_cpu_baseline(model, args.cpu_seconds)
    return {
        "metric": METRIC, "value": round(world * batch / (step_ms * 1e-3), 1), "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "s8xs8->s32",
        "data": "synthetic (seeded splitmix64 input images; seeded random-init int8 weights)",
        "config": {"workload": f"{net} int8 forward, chained (stem, max pool, convs with fused residual adds, "
                               f"global average pool), per-GPU batch {batch}",
                   "global_batch": batch * world, "per_gpu_batch": batch, "parallelism": f"dp{world} (batch shards)",
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
        "tops_per_gpu": round(ops / (step_ms * 1e-3) / 1e12, 1),
        "frac_of_int8_peak": round(ops / (step_ms * 1e-3) / 1e12 / (2.0 * peaks["bf16_tflops"]), 4),
        "gpu_launches": int(launches), "clocks": clocks,
        "verify": {"pooled_feature_checksum_per_rank": checksums},
        **({"cpu_baseline": cpu} if cpu else {}),
    }


def chain_cpu_baseline(model, budget_s: float) -> dict:
    """The same chained forward on the host cores: the C oracle's threaded int8 conv plus its
    requant / residual / pool restatements, on a bounded sample of images."""
    from my_own_cnn_b200 import nets, synth
    from oracle import oracle

    threads = oracle.cpu_threads()

    def forward(img0: int, nimg: int):
        bufs = {0: synth.s8_table_host(SEED, 1, nets.act_table(), img0 * 224 * 224 * 3,
                                       nimg * 224 * 224 * 3).reshape(nimg, 224, 224, 3)}
        for op in model.plan:
            src = bufs[op.src]
            if op.kind == "conv":
                sp = model.specs[op.layer]
                w, b, s = (t.cpu().numpy() for t in model.weights[op.layer])
                a = oracle.conv_args(nimg, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride,
                                     groups=sp.groups)
                acc = oracle.conv_s8(a, src, w, threads=threads)
                lo, hi = (-128, 127) if sp.linear else ((0, nets.Q6) if sp.relu6 else (0, 127))
                bufs[op.dst] = (oracle.requant_res_s8(acc, b, s, bufs[op.res], nets.RES_SCALE, 0, lo, hi)
                                if op.res >= 0 else oracle.requant_s8(acc, b, s, 0, lo, hi))
            elif op.kind == "maxpool":
                bufs[op.dst] = oracle.maxpool_s8(src, 3, 3, 2, 2, 1, 1)
            else:
                bufs[op.dst] = oracle.global_avgpool_s8(src)

    t0 = time.perf_counter()
    forward(0, 1)
    t_one = time.perf_counter() - t0
    images = int(max(1, min(64, budget_s / max(t_one, 1e-3))))
    t0 = time.perf_counter()
    forward(0, images)
    dt = time.perf_counter() - t0
    return {"value": round(images / dt, 3), "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"{images} images through the whole chained {model.name} forward; C oracle conv "
                      f"(threaded over output pixels) + requant / residual / pool restatements",
            "seconds": round(dt, 2)}


def run_bmm(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Config 2: batch 64 of 1024^3 int8 NN GEMMs per GPU, int32 accumulators and the per-column
    requantized int8 variant (two launches per step)."""
    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import synth
    from my_own_cnn_b200.shard import max_over_ranks

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    batch, M = 64, 1024
    A = synth.fill_s8_uniform(torch.empty((batch, M, M), dtype=torch.int8, device=dev), SEED + rank, 101)
    B = synth.fill_s8_uniform(torch.empty((batch, M, M), dtype=torch.int8, device=dev), SEED + rank, 102)
    sc = torch.from_numpy(synth.scales_f32(M, SEED, 103)).to(dev)
    C32 = torch.empty((batch, M, M), dtype=torch.int32, device=dev)
    C8 = torch.empty((batch, M, M), dtype=torch.int8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    e32, e8 = b2q.Epilogue.int32(), b2q.Epilogue.int8()
    for _ in range(args.warmup):
        b2q.bmm_s8_into(C32, A, B, None, None, batch, M, M, M, 0, 0, e32)
        b2q.bmm_s8_into(C8, A, B, None, sc, batch, M, M, M, 0, 0, e8)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    torch.cuda.synchronize()
    for st in range(args.steps):
        flush.fill_(st & 0x7F)
        ev[st][0].record(stream)
        b2q.bmm_s8_into(C32, A, B, None, None, batch, M, M, M, 0, 0, e32)
        ev[st][1].record(stream)
        b2q.bmm_s8_into(C8, A, B, None, sc, batch, M, M, M, 0, 0, e8)
        ev[st][2].record(stream)
    torch.cuda.synchronize()
    t32 = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    t8 = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    # The reference's own entry (bmm_matmul_i32 on int32 operands holding the same int8 values):
    # the tensor-core route (int8 copies + tcgen05 GEMM), and one call forced onto the CUDA-core kernel.
    A32, B32 = A.to(torch.int32), B.to(torch.int32)
    del flush
    def time_i32(reps):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
        torch.cuda.synchronize()
        evs[0].record(stream)
        for i in range(reps):
            b2q.bmm_matmul_i32(A32, B32, C32, batch, M, M, M, 0, 0)
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
        return sum(evs[i].elapsed_time(evs[i + 1]) for i in range(reps)) / reps
    time_i32(3)
    ti32 = time_i32(args.steps)
    b2q.set_path_policy(1)
    try:
        ti32_cc = time_i32(1)
    finally:
        b2q.set_path_policy(0)
    del A32, B32
    t32, t8, ti32, ti32_cc = max_over_ranks([t32, t8, ti32, ti32_cc], device=dev)
    if rank != 0:
        return None
    peaks = load_peaks()
    ops = 2 * batch * M ** 3
    bytes32 = 2 * batch * M * M + 4 * batch * M * M
    return {"metric": "int8 bmm TOPS/GPU (config 2)", "value": round(world * 2 * ops / ((t32 + t8) * 1e-3) / 1e12, 1),
            "unit": "TOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t32 + t8, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "s8xs8->s32", "data": "synthetic (seeded splitmix64)",
            "config": {"workload": "config2 bmm batch 64, M=N=K=1024, NN, int32 out + per-column int8 requant out"},
            "int32_out": {"ms": round(t32, 4), "tops": round(ops / t32 / 1e9, 1),
                          "hbm_gbs": round(bytes32 / t32 / 1e6, 1), "hbm_frac": round(bytes32 / t32 / 1e6 / peaks["hbm_gbs"], 4)},
            "int8_out": {"ms": round(t8, 4), "tops": round(ops / t8 / 1e9, 1),
                         "frac_of_int8_peak": round(ops / t8 / 1e9 / (2 * peaks["bf16_tflops"]), 4)},
            "dropin_bmm_matmul_i32": {"ms": round(ti32, 4), "tops": round(ops / ti32 / 1e9, 1),
                                      "cuda_core_ms": round(ti32_cc, 4),
                                      "note": "int32 operands (int8 values): int8 copies + tcgen05 GEMM; "
                                              "cuda_core_ms = the same call forced onto the CUDA-core kernel, "
                                              "no L2 flush (inputs 512 MiB > L2)"}}


# ------------------------------------------------------------- per-config sub-records (N = 1)

SUB_KEEP = ("value", "unit", "ms_per_step", "steps", "warmup", "tops_per_gpu", "frac_of_int8_peak", "by_path",
            "roofline", "roofline_depthwise", "slowest_layers", "cpu_baseline", "int32_out", "int8_out", "config",
            "dropin_bmm_matmul_i32",
            "gpu_launches", "clocks")


def _trim(rec: dict) -> dict:
    out = {k: rec[k] for k in SUB_KEEP if k in rec}
    if "config" in out:
        out["workload"] = out.pop("config").get("workload")
    return out


def _timed_ms(fn, steps: int, flush, stream) -> list[float]:
    """Per-step CUDA-event times of fn on `stream`, L2 flushed between steps outside the events."""
    import torch

    out = []
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i, (a, b) in enumerate(evs):
        flush.fill_(i & 0x7F)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def _roof(ops: float, nbytes: float, ms: float, peaks: dict) -> dict:
    """Binding roof of one launch: the slower of the int8 tensor time and the HBM time."""
    int8_peak = 2.0 * peaks["bf16_tflops"]
    t_tensor = ops / (int8_peak * 1e12) * 1e3
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
    bound = "tensor" if t_tensor >= t_hbm else "hbm"
    if bound == "tensor":
        ach, peak, unit = ops / (ms * 1e-3) / 1e12, int8_peak, "TOP/s"
    else:
        ach, peak, unit = nbytes / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
    return {"bound": bound, "achieved": round(ach, 2), "peak": round(peak, 1), "unit": unit,
            "frac": round(ach / peak, 4), "roof_ms": round(max(t_tensor, t_hbm), 5),
            "peak_source": peaks["source"]}


def _graph_us(fn, dev, calls: int = 100) -> float | None:
    """Device time per call of `fn` when `calls` calls are captured in one CUDA graph and replayed
    (no host work between the kernels), min of 5 replays; None if the capture is refused."""
    import torch

    side = torch.cuda.Stream(dev)
    try:
        g = torch.cuda.CUDAGraph()
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=side):
                for _ in range(calls):
                    fn()
        torch.cuda.synchronize()
        best = None
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            t = a.elapsed_time(b) * 1e3 / calls
            best = t if best is None else min(best, t)
        return round(best, 3)
    except Exception as ex:  # capture not possible on this path: report it, do not fail the bench
        torch.cuda.synchronize()
        return f"capture failed: {type(ex).__name__}"


def run_config1(args, dev) -> dict:
    """one conv, 1x56x56x64, 3x3 pad 1, K = 64, bias + per-channel requant to int8.
    Also the reference-API drop-in (launch_fprop_nhwc_qi32, float codes, U8 zero points) at the same
    geometry, and both back to back without an L2 flush (the latency a caller sees in a loop)."""
    import numpy as np
    import torch

    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import synth

    n, h, w, c, k = 1, 56, 56, 64, 64
    p = b2q.Conv2DParams()
    x = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device=dev), SEED, 201)
    wt = synth.fill_s8_uniform(torch.empty((k, 3, 3, c), dtype=torch.int8, device=dev), SEED, 202)
    b = synth.fill_i32_uniform(torch.empty(k, dtype=torch.int32, device=dev), SEED, 203, -2**15, 2**15)
    sc = torch.from_numpy(synth.scales_f32(k, SEED, 204)).to(dev)
    y = torch.empty((n, h, w, k), dtype=torch.int8, device=dev)
    epi = b2q.Epilogue.int8()
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    run = lambda: b2q.conv2d_s8_into(y, x, wt, b, sc, n, h, w, c, 3, 3, k, p, epi)
    for _ in range(args.warmup):
        run()
    path = b2q.last_path()
    steps = max(args.steps, 20)
    ms = statistics.median(_timed_ms(run, steps, flush, stream))
    hot = _timed_ms(lambda: [run() for _ in range(100)], 3, flush, stream)
    hot_us = min(hot) * 10.0
    graph_us = _graph_us(run, dev)
    # drop-in: U8 float codes (x + 127 in [0, 254]), per-image zero point 91, filter zero point 37
    xf = (x.float() + 127.0).contiguous()
    wf = (wt.float() + 127.0).contiguous()
    y32 = torch.empty((n, h, w, k), dtype=torch.int32, device=dev)
    qin = b2q.qparams_to_device([b2q.QuantizationParametersU8(91, 0.25)])
    qf = b2q.qparams_to_device([b2q.QuantizationParametersU8(37, 0.5)])
    drop = lambda: b2q.launch_fprop_nhwc_qi32(xf, wf, y32, n, h, w, c, 3, 3, k, p, qin, qf)
    for _ in range(args.warmup):
        drop()
    dpath = b2q.last_path()
    dms = statistics.median(_timed_ms(drop, steps, flush, stream))
    dhot = min(_timed_ms(lambda: [drop() for _ in range(100)], 3, flush, stream)) * 10.0
    dgraph_us = _graph_us(drop, dev)
    peaks = load_peaks()
    ops = 2 * n * h * w * k * 9 * c
    nbytes = n * h * w * c + k * 9 * c + n * h * w * k + 8 * k
    rec = {"workload": "config1 conv 1x56x56x64 3x3/1 p1 K64, bias+per-channel requant int8",
           "value": round(1.0 / (ms * 1e-3), 1), "unit": "images/s", "ms_per_step": round(ms, 5), "steps": steps,
           "path": path, "tops": round(ops / ms / 1e9, 2), "back_to_back_us": round(hot_us, 2),
           "graph_us": graph_us,
           "roofline": _roof(ops, nbytes, ms, peaks),
           "note": "M = 3136 rows: 28 row tiles on 148 SMs; latency-bound (roof_ms is the tensor/HBM roof). "
                   "back_to_back_us: 100 calls from Python in a row (includes the host call path); graph_us: the "
                   "same 100 calls captured once in a CUDA graph and replayed (device time per conv)",
           "dropin_qi32": {"entry": "launch_fprop_nhwc_qi32 (U8 float codes, zero points 91 / 37)", "path": dpath,
                           "ms_per_step": round(dms, 5), "back_to_back_us": round(dhot, 2),
                           "graph_us": dgraph_us,
                           "roofline": _roof(ops, 4 * (n * h * w * c + k * 9 * c + n * h * w * k), dms, peaks)}}
    if not args.no_cpu_baseline:
        from oracle import oracle

        xs, ws_ = x.cpu().numpy().astype(np.float32), wt.cpu().numpy().astype(np.float32)
        bh, sh = b.cpu().numpy(), sc.cpu().numpy()
        a = oracle.conv_args(n, h, w, c, 3, 3, k)
        use_ref = oracle.ref_available()
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0) or reps == 0:
            acc = (oracle.ref_conv_qi32(a, 1, xs, ws_, np.zeros(1, np.int32), 0, False) if use_ref
                   else oracle.conv_s8(a, x.cpu().numpy(), wt.cpu().numpy()))
            oracle.requant_s8(acc, bh, sh)
            reps += 1
        dt = time.perf_counter() - t0
        rec["cpu_baseline"] = {"value": round(reps / dt, 3), "unit": "images/s", "cores": 1,
                               "kind": "reference" if use_ref else "port",
                               "sample": f"the whole conv (one image) {reps} times; src/cpu_ref.cpp cpu_fprop_nhwc_qi32 "
                                         "+ CPU requant, one thread (one image does not split over images)"}
    return rec


def net_cpu_baseline(name: str, batch: int, budget_s: float) -> dict:
    """Configs 3 / 5 per layer on the host cores: the reference's cpu_fprop_nhwc_qi32 (float codes,
    zero points 0) + the CPU requant for every layer of the table, images split over threads."""
    import numpy as np

    from my_own_cnn_b200 import nets
    from oracle import oracle

    threads = oracle.cpu_threads()
    specs = nets.NETS[name]()
    use_ref = oracle.ref_available()
    rng = np.random.default_rng(7)

    def run(images: int) -> float:
        total = 0.0
        for sp in specs:
            x = rng.integers(0, 128, size=(images, sp.h, sp.w, sp.c)).astype(np.int8)
            w = rng.integers(-127, 128, size=(sp.k, sp.r, sp.r, sp.c // sp.groups)).astype(np.int8)
            b = rng.integers(-2**15, 2**15, size=sp.k).astype(np.int32)
            s = np.full(sp.k, 5e-4, np.float32)
            a = oracle.conv_args(images, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride,
                                 groups=sp.groups)
            xf, wf = x.astype(np.float32), w.astype(np.float32)
            t0 = time.perf_counter()
            acc = oracle.ref_conv_qi32_threaded(a, xf, wf, threads) if use_ref else oracle.conv_s8(a, x, w, threads)
            oracle.requant_s8(acc, b, s, 0, 0, 127)
            total += time.perf_counter() - t0
        return total

    t_probe = run(1)
    images = threads
    if t_probe * images / threads * 1.2 > budget_s:
        images = max(1, int(budget_s / t_probe))
    dt = run(images)
    return {"value": round(images / dt, 3), "unit": "images/s", "cores": threads,
            "kind": "reference" if use_ref else "port",
            "sample": f"{images} images (of {batch}) through every conv of the {name} table, fresh inputs per layer; "
                      f"src/cpu_ref.cpp cpu_fprop_nhwc_qi32 on float codes + CPU requant, images split over "
                      f"{threads} threads", "seconds": round(dt, 2)}


def bmm_cpu_baseline(budget_s: float) -> dict:
    import numpy as np

    from oracle import oracle

    threads = oracle.cpu_threads()
    M = 1024
    rng = np.random.default_rng(3)
    A = rng.integers(-127, 128, size=(1, M, M)).astype(np.int8)
    B = rng.integers(-127, 128, size=(1, M, M)).astype(np.int8)
    t0 = time.perf_counter()
    oracle.bmm_s8(A, B, 1, M, M, M, 0, 0, 1)
    t_one = time.perf_counter() - t0
    items = max(threads, min(64, int(budget_s / max(t_one, 1e-3)) * threads // threads))
    items = max(threads, items // threads * threads)
    A = rng.integers(-127, 128, size=(items, M, M)).astype(np.int8)
    B = rng.integers(-127, 128, size=(items, M, M)).astype(np.int8)
    t0 = time.perf_counter()
    oracle.bmm_s8(A, B, items, M, M, M, 0, 0, threads)
    dt = time.perf_counter() - t0
    ops = 2.0 * items * M ** 3
    return {"value": round(ops / dt / 1e12, 5), "unit": "TOP/s", "cores": threads, "kind": "port",
            "sample": f"{items} of the 64 batch items (int32 out), restated CPU GEMM (bmm.h:9-29) over {threads} "
                      f"threads", "seconds": round(dt, 2)}


def run_subconfigs(args, dev) -> dict:
    """Every other BASELINE config at N = 1, each as a sub-record of the default line."""
    import copy

    import torch

    sub_steps = max(5, min(args.steps, 20))
    out = {}

    def sub(config: str, fn):
        a = copy.copy(args)
        a.config, a.steps, a.warmup, a.batch, a.layers = config, sub_steps, 3, 0, ""
        a.cpu_seconds = args.sub_cpu_seconds
        a.no_cpu_baseline = True
        try:
            rec = _trim(fn(a, 0, 1, dev.index or 0))
        finally:
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
        return rec

    a1 = copy.copy(args)
    a1.cpu_seconds = args.sub_cpu_seconds
    out["config1"] = run_config1(a1, dev)
    torch.cuda.empty_cache()
    out["config2_bmm"] = sub("bmm", run_bmm)
    out["config3_resnet50_layers"] = sub("resnet50", run_net)
    out["config3_resnet50_chain"] = sub("resnet50-chain", run_chain)
    out["config5_mobilenetv2_layers"] = sub("mobilenetv2", run_net)
    out["config5_mobilenetv2_chain"] = sub("mobilenetv2-chain", run_chain)
    if not args.no_cpu_baseline:
        from my_own_cnn_b200 import nets

        out["config2_bmm"]["cpu_baseline"] = bmm_cpu_baseline(args.sub_cpu_seconds)
        out["config3_resnet50_layers"]["cpu_baseline"] = net_cpu_baseline("resnet50", 256, args.sub_cpu_seconds)
        out["config5_mobilenetv2_layers"]["cpu_baseline"] = net_cpu_baseline("mobilenetv2", 512, args.sub_cpu_seconds)
        model_dev = torch.device("cuda", dev.index or 0)
        for key, name in (("config3_resnet50_chain", "resnet50"), ("config5_mobilenetv2_chain", "mobilenetv2")):
            out[key]["cpu_baseline"] = chain_cpu_baseline(nets.ChainedNet(name, SEED, model_dev), args.sub_cpu_seconds)
            torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"],
                    help="reference = the reference's CPU path (the reference arm); reference-gpu = the reference's "
                         "own CUDA quantized conv against this library's drop-in (secondary baseline)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--sustain-s", type=float, default=1.5,
                    help="seconds of back-to-back headline steps with clocks sampled (0 = off)")
    ap.add_argument("--sub-cpu-seconds", type=float, default=6.0, help="CPU budget of each sub-record's baseline")
    ap.add_argument("--no-subconfigs", action="store_true",
                    help="N=1: skip the per-config sub-records (configs 1, 2, 3, 5) of the default line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunk", type=int, default=64, help="images per chunk of the e2e pipeline")
    ap.add_argument("--config", default="pointwise",
                    choices=["pointwise", "resnet50", "mobilenetv2", "resnet50-chain", "mobilenetv2-chain", "bmm"],
                    help="pointwise (BASELINE config 4, the default bench line); the others report configs 3 / 5 / 2")
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch for the network configs (0 = BASELINE)")
    ap.add_argument("--layers", default="", help="regex on layer names: run only those layers of resnet50 / "
                    "mobilenetv2 (profiling a single layer; the default runs the whole table)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return
    if args.impl == "reference-gpu":
        if rank != 0:
            return
        for rec in run_reference_gpu(args):
            print(json.dumps(rec), flush=True)
        return

    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    if args.config in NET_BATCH:
        out = run_net(args, rank, world, local_rank)
    elif args.config.endswith("-chain"):
        out = run_chain(args, rank, world, local_rank)
    elif args.config == "bmm":
        out = run_bmm(args, rank, world, local_rank)
    else:
        out = run_ours(args, rank, world, local_rank)
        if world == 1 and not args.no_subconfigs and out is not None:
            import torch

            out["configs"] = run_subconfigs(args, torch.device("cuda", local_rank))
    if out is not None:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
