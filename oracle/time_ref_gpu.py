"""Secondary baseline (test / measurement infrastructure): the reference's own CUDA quantized conv
(src/cuda_kernels.cu:1336-1392 -- per-call workspace cudaMalloc/cudaFree, im2col to int32,
32x32-tile SIMT int32 GEMM, unpack; compiled unmodified into oracle/_ref/libref_gpu.so) timed on
the same B200 as this library's int8 tensor-core conv, on BASELINE configs 1 and 4 (int32
accumulator outputs, zero points 0).  Also checks that both produce identical accumulators.

Usage: python oracle/time_ref_gpu.py   (prints one JSON line per case)
"""
from __future__ import annotations

import ctypes
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import my_own_cnn_b200 as b2q  # noqa: E402
from my_own_cnn_b200 import synth  # noqa: E402

LIB = Path(__file__).resolve().parent / "_ref" / "libref_gpu.so"


def timed(fn, iters, flush):
    fn()
    torch.cuda.synchronize()
    ts = []
    for i in range(iters):
        flush.fill_(i & 0x7F)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return sorted(ts)[len(ts) // 2]


def main():
    ref = ctypes.CDLL(str(LIB))
    ref.refgpu_fprop_qi32_s5.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 9 + [ctypes.c_void_p] * 2
    flush = torch.empty(256 << 20, dtype=torch.int8, device="cuda")
    cases = [("config1 3x3 N1 56x56 C64->K64", 1, 56, 56, 64, 3, 64, 1, 1),
             ("config4a 1x1 b512 14x14 C1024->K2048", 512, 14, 14, 1024, 1, 2048, 0, 1),
             ("config4b 1x1 b512 14x14 C2048->K512", 512, 14, 14, 2048, 1, 512, 0, 1)]
    for name, n, h, w, c, r, k, pad, st in cases:
        x8 = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device="cuda"), 42, 1)
        w8 = synth.fill_s8_uniform(torch.empty((k, r, r, c), dtype=torch.int8, device="cuda"), 42, 2)
        xf, wf = x8.float(), w8.float()
        p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, 1)
        ho, wo = b2q.conv_out_shape(h, w, c, r, r, k, p)
        y_ref = torch.empty((n, ho, wo, k), dtype=torch.int32, device="cuda")
        y_me = torch.empty_like(y_ref)
        qp_in = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)] * n)
        qp_f = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)])

        def run_ref():
            rc = ref.refgpu_fprop_qi32_s5(xf.data_ptr(), wf.data_ptr(), y_ref.data_ptr(), n, h, w, c, r, r, k, pad, st,
                                          qp_in.data_ptr(), qp_f.data_ptr())
            assert rc == 0

        def run_me():
            b2q.conv2d_s8_into(y_me, x8, w8, None, None, n, h, w, c, r, r, k, p, b2q.Epilogue.int32())

        t_ref = timed(run_ref, 3, flush)
        t_me = timed(run_me, 20, flush)
        ops = 2 * n * ho * wo * k * r * r * c
        print(json.dumps({"case": name, "reference_gpu_ms": round(t_ref, 4), "reference_gpu_tops": round(ops / t_ref / 1e9, 2),
                          "b200q_ms": round(t_me, 4), "b200q_tops": round(ops / t_me / 1e9, 1),
                          "b200q_path": b2q.last_path(), "speedup": round(t_ref / t_me, 1),
                          "identical_int32": bool(torch.equal(y_ref, y_me))}), flush=True)


if __name__ == "__main__":
    main()
