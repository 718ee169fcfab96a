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
        "config": {"workload": "config4 pointwise 1x1 pair: b512 14x14 C1024->K2048 then C2048->K512, "
                               "bias+per-channel requant int8 epilogue",
                   "global_batch": BATCH * world, "per_gpu_batch": BATCH, "parallelism": f"dp{world} (batch shards)",
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
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
        "verify": {"checksums_y2_y1_per_rank": checksums},
    }
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    return out


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
        "config": {"workload": "config4 pointwise 1x1 pair: b512 14x14 C1024->K2048 then C2048->K512, "
                               "bias+per-channel requant int8 epilogue", "per_step_sample_images": images},
        "impl": "reference",
        "cpu_baseline": {"value": round(val, 3), "unit": "images/s", "cores": threads, "kind": kind,
                         "sample": f"{images} images per step, images split over {threads} threads"},
        "e2e": {"value": round(val, 3), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


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
    t32, t8 = max_over_ranks([t32, t8], device=dev)
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
                         "frac_of_int8_peak": round(ops / t8 / 1e9 / (2 * peaks["bf16_tflops"]), 4)}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
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
    if out is not None:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
