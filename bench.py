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
    assert b2q.last_path() == "tcgen05-tiled", b2q.last_path()
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
                     "kernel": "tc_gemm_s8_kernel",
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunk", type=int, default=64, help="images per chunk of the e2e pipeline")
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
    out = run_ours(args, rank, world, local_rank)
    if out is not None:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
