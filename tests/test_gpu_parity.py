"""GPU parity tests: every kernel family against the CPU oracle, through the C ABI.

Bar: bit-exact for int32 accumulators and int8 requantized outputs; the fp32 dequantized output
is compared with a relative tolerance of 1e-5 (it is in fact computed by the same IEEE ops)."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.kat import kat_cases, rng_s8

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
FP32_RTOL = 1e-5


def _b2q():
    import my_own_cnn_b200 as b2q

    return b2q


def _qparams(kind, zps):
    b2q = _b2q()
    if kind == 0:
        return [b2q.QuantizationParametersU8(int(z) & 0xFF, 0.25) for z in zps]
    return [b2q.QuantizationParametersS5(int(z), 31, 0.5) for z in zps]


# ------------------------------------------------------------------ drop-in (reference API)

def test_dropin_qi32_known_answers(cuda_lib, golden):
    b2q = _b2q()
    for kc in kat_cases(golden):
        dev = torch.device("cuda")
        x = torch.from_numpy(kc.x.reshape(-1)).to(dev)
        w = torch.from_numpy(kc.wt.reshape(-1)).to(dev)
        y = torch.full(kc.y.shape, 0x7EADBEEF, dtype=torch.int32, device=dev)
        in_qp = b2q.qparams_to_device(_qparams(kc.kind, kc.zp_in))
        f_qp = b2q.qparams_to_device(_qparams(kc.kind, [kc.zp_f]))
        qt = b2q.DataType.LinQuantU8 if kc.kind == 0 else b2q.DataType.LinQuantS5
        p = b2q.Conv2DParams(kc.pad_h, kc.pad_w, kc.stride_h, kc.stride_w, kc.dil_h, kc.dil_w, kc.groups)
        if kc.blocked:
            b2q.launch_block_fprop_nhwc_qi32(x, w, y, kc.n, kc.h, kc.w, kc.c, kc.r, kc.s, kc.k,
                                             b2q.BlockConv2DParams(p, kc.by, kc.bx), in_qp, f_qp, qtype=qt)
        else:
            b2q.launch_fprop_nhwc_qi32(x, w, y, kc.n, kc.h, kc.w, kc.c, kc.r, kc.s, kc.k, p, in_qp, f_qp, qtype=qt)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), kc.y, err_msg=kc.name)


def test_reference_quant_conv_test_links_and_passes(cuda_lib):
    """The reference's unmodified quant_conv_test.cu, linked against the shim (no reference kernels)."""
    binary = ROOT / "oracle" / "_ref" / "quant_conv_test_b200"
    if not binary.exists():
        pytest.skip("reference test binary not built (needs the reference sources at build time)")
    proc = subprocess.run([str(binary)], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "quant_conv_test passed" in proc.stdout


def test_dropin_rejects_null_qparams(cuda_lib):
    b2q = _b2q()
    x = torch.zeros(16, device="cuda")
    y = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="non-null quantization parameters"):
        b2q.launch_fprop_nhwc_qi32(x, x, y, 1, 2, 2, 4, 1, 1, 4, b2q.Conv2DParams(0, 0), None, None)


def test_bmm_matmul_i32_exact_wraparound(cuda_lib):
    b2q = _b2q()
    rng = np.random.default_rng(11)
    for ta in (0, 1):
        for tb in (0, 1):
            for batch, M, N, K in [(1, 1, 1, 1), (2, 17, 19, 13), (3, 64, 70, 33)]:
                A = rng.integers(-2**31, 2**31, size=(batch, K, M) if ta else (batch, M, K), dtype=np.int64).astype(np.int32)
                B = rng.integers(-2**31, 2**31, size=(batch, N, K) if tb else (batch, K, N), dtype=np.int64).astype(np.int32)
                C = torch.empty((batch, M, N), dtype=torch.int32, device="cuda")
                b2q.bmm_matmul_i32(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C, batch, M, N, K, ta, tb)
                torch.cuda.synchronize()
                np.testing.assert_array_equal(C.cpu().numpy(), oracle.bmm_i32(A, B, batch, M, N, K, ta, tb))


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_bmm_matmul_i32_tensor_core_route(cuda_lib, ta, tb):
    """int32 operands whose values fit int8 take the tcgen05 route (path 16), bit-exact; one value
    outside [-128, 127] anywhere in A or B makes the device-side fallback recompute C exactly."""
    b2q = _b2q()
    rng = np.random.default_rng(23 + 2 * ta + tb)
    for batch, M, N, K in [(1, 16, 16, 16), (3, 144, 80, 96), (2, 208, 272, 400), (2, 256, 512, 1040)]:
        A = rng.integers(-128, 128, size=(batch, K, M) if ta else (batch, M, K)).astype(np.int32)
        B = rng.integers(-128, 128, size=(batch, N, K) if tb else (batch, K, N)).astype(np.int32)
        want = oracle.bmm_i32(A, B, batch, M, N, K, ta, tb)
        for poison in (None, "A", "B"):
            Ap, Bp = A.copy(), B.copy()
            if poison == "A":
                Ap.reshape(-1)[Ap.size // 2 + 1] = 300
            if poison == "B":
                Bp.reshape(-1)[-1] = -129
            exp = want if poison is None else oracle.bmm_i32(Ap, Bp, batch, M, N, K, ta, tb)
            C = torch.full((batch, M, N), 7, dtype=torch.int32, device="cuda")
            b2q.bmm_matmul_i32(torch.from_numpy(Ap).cuda(), torch.from_numpy(Bp).cuda(), C, batch, M, N, K, ta, tb)
            torch.cuda.synchronize()
            assert b2q.last_path() == "tcgen05-bmm-i32"
            np.testing.assert_array_equal(C.cpu().numpy(), exp)


def test_bmm_matmul_i32_config2_full_size_sampled(cuda_lib):
    """BASELINE config 2 (64 x 1024^3) through the int32 drop-in with int8-range values: the tensor-core
    route, two sampled batches checked against the oracle."""
    b2q = _b2q()
    batch, M, N, K = 64, 1024, 1024, 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randint(-127, 128, (batch, M, K), dtype=torch.int32, device="cuda", generator=g)
    B = torch.randint(-127, 128, (batch, K, N), dtype=torch.int32, device="cuda", generator=g)
    C = torch.empty((batch, M, N), dtype=torch.int32, device="cuda")
    b2q.bmm_matmul_i32(A, B, C, batch, M, N, K, 0, 0)
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-bmm-i32"
    for b in (0, 41):
        want = oracle.bmm_i32(A[b:b + 1].cpu().numpy(), B[b:b + 1].cpu().numpy(), 1, M, N, K, 0, 0)
        np.testing.assert_array_equal(C[b:b + 1].cpu().numpy(), want)


# ------------------------------------------------------------------ int8 conv

def _conv_case(n, h, w, c, r, s, k, p, seed, epi_kind="all", groups=1):
    """Run conv2d_s8 for each epilogue and compare with the oracle; returns the dispatched paths."""
    b2q = _b2q()
    x = rng_s8(seed, (n, h, w, c))
    wt = rng_s8(seed + 1, (k, r, s, c // groups))
    rng = np.random.default_rng(seed + 2)
    bias = rng.integers(-2**15, 2**15 + 1, size=k).astype(np.int32)
    scale = rng.uniform(1e-4, 1e-3, size=k).astype(np.float32)
    a = oracle.conv_args(n, h, w, c, r, s, k, p.pad_h, p.pad_w, p.stride_h, p.stride_w, p.dilation_h,
                         p.dilation_w, groups)
    acc = oracle.conv_s8(a, x, wt, threads=4)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
    bd, sd = torch.from_numpy(bias).cuda(), torch.from_numpy(scale).cuda()
    paths = set()
    kinds = ["s32", "s8", "relu", "f32"] if epi_kind == "all" else [epi_kind]
    for kind in kinds:
        if kind == "s32":
            y = b2q.conv2d_s8(xd, wd, None, None, p, b2q.Epilogue.int32())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(y.cpu().numpy(), acc)
        elif kind == "s8":
            y = b2q.conv2d_s8(xd, wd, bd, sd, p, b2q.Epilogue.int8())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(y.cpu().numpy(), oracle.requant_s8(acc, bias, scale))
        elif kind == "relu":
            y = b2q.conv2d_s8(xd, wd, bd, sd, p, b2q.Epilogue.int8(relu6_q=97))
            torch.cuda.synchronize()
            np.testing.assert_array_equal(y.cpu().numpy(), oracle.requant_s8(acc, bias, scale, 0, 0, 97))
        else:
            y = b2q.conv2d_s8(xd, wd, bd, sd, p, b2q.Epilogue.fp32())
            torch.cuda.synchronize()
            np.testing.assert_allclose(y.cpu().numpy(), oracle.dequant_f32(acc, bias, scale), rtol=FP32_RTOL, atol=0)
        paths.add(b2q.last_path())
        # the host-side plan (no launch) names the kernel family the call dispatched to
        epi = {"s32": b2q.Epilogue.int32(), "s8": b2q.Epilogue.int8(), "relu": b2q.Epilogue.int8(relu6_q=97),
               "f32": b2q.Epilogue.fp32()}[kind]
        assert b2q.conv2d_s8_plan(n, h, w, c, r, s, k, p, epi) == b2q.last_path(), kind
    return paths


@pytest.mark.parametrize("shape", [
    # n, h, w, c, r, s, k, pad, stride, dil
    (4, 14, 14, 256, 3, 3, 256, 1, 1, 1),  # ResNet stage-3 3x3 (C = 256: no row tiles)
    (2, 34, 34, 64, 3, 3, 80, 1, 2, 1),    # stride 2, K edge (80 = 64 + 16)
    (1, 40, 36, 96, 3, 3, 48, 2, 1, 2),    # dilation 2, BK 32 chunks
    (2, 24, 24, 256, 1, 1, 272, 0, 2, 1),  # 1x1 stride 2 (projection shortcut) through im2col
    (1, 64, 64, 32, 5, 5, 32, 2, 1, 1),    # 5x5, C = 32
    (2, 96, 96, 16, 3, 3, 24, 1, 1, 1),    # C = 16 (zero-filled half K block), K = 24 (scalar stores)
    (2, 30, 30, 144, 3, 3, 144, 1, 2, 1),  # C = 144 = 4.5 x 32 (MobileNetV2 expand width), stride 2
    (2, 40, 40, 48, 3, 3, 64, 1, 1, 1),    # C = 48
])
def test_conv_s8_tcgen05_im2col(cuda_lib, shape):
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st, dil = shape
    p = b2q.Conv2DParams(pad, pad, st, st, dil, dil, 1)
    paths = _conv_case(n, h, w, c, r, s, k, p, seed=sum(shape))
    assert paths == {"tcgen05-im2col"}, paths


@pytest.mark.parametrize("shape", [
    (2, 14, 14, 1024, 256),  # config 4 shape family, small batch
    (1, 14, 14, 512, 2048),
    (3, 7, 9, 64, 16),       # M edge (189 rows), tiny N
    (1, 13, 11, 160, 96),    # BK 32 chunks, N edge
    (4, 28, 28, 16, 96),     # C = 16 (MobileNetV2 expand 16 -> 96)
    (2, 28, 28, 144, 24),    # C = 144, K = 24 (project 144 -> 24)
])
def test_conv_s8_tcgen05_pointwise(cuda_lib, shape):
    b2q = _b2q()
    n, h, w, c, k = shape
    p = b2q.Conv2DParams(0, 0, 1, 1, 1, 1, 1)
    paths = _conv_case(n, h, w, c, 1, 1, k, p, seed=sum(shape))
    # narrow layers whose rows group into G pixels (G * K <= 256, G * C <= 256, G | M) run pixel-grouped
    grouped = any(g * k <= 256 and g * c <= 256 and (g * c) % 16 == 0 and (n * h * w) % g == 0 for g in (2, 4, 8, 16))
    assert paths == {"tcgen05-tiled-grouped" if grouped else "tcgen05-tiled"}, paths


@pytest.mark.parametrize("shape,groups,expect", [
    # C % 16 == 0 depthwise: int8 outputs take the TMA-staged kernel, int32 / fp32 the register one
    ((2, 20, 20, 48, 3, 3, 48, 1, 2, 1), 48, "cuda-core-depthwise|cuda-core-depthwise-tma"),   # s2
    ((1, 17, 19, 96, 3, 3, 96, 1, 1, 1), 96, "cuda-core-depthwise|cuda-core-depthwise-tma"),   # W tails
    ((2, 9, 10, 8, 3, 3, 8, 1, 2, 1), 8, "cuda-core-depthwise"),        # C = 8, s2, 2-pixel groups
    ((3, 7, 7, 960, 3, 3, 960, 1, 1, 1), 960, "cuda-core-depthwise|cuda-core-depthwise-tma"),  # 7x7 stage
    ((1, 11, 13, 16, 3, 3, 16, 2, 1, 2), 16, "cuda-core-depthwise"),    # dilation 2: one pixel/thread
    ((2, 23, 23, 3, 7, 7, 64, 3, 2, 1), 1, "cuda-core-generic"),      # stem C = 3
    ((1, 11, 13, 24, 1, 1, 40, 0, 1, 1), 1, "cuda-core-generic"),     # C % 16 != 0, odd M: no pixel grouping
    ((1, 12, 12, 24, 1, 1, 40, 0, 1, 1), 1, "tcgen05-tiled-grouped"),  # C % 16 != 0: 4-pixel rows of 96 B
    ((2, 9, 9, 32, 3, 3, 64, 1, 1, 1), 2, "cuda-core-generic"),       # grouped
    ((1, 6, 6, 48, 3, 3, 64, 1, 1, 1), 1, "cuda-core-generic"),       # tiny tensor (36 output rows)
    ((2, 14, 14, 256, 3, 3, 256, 1, 1, 1), 1, "tcgen05-packed"),      # < 128 KiB: packed, not im2col
])
def test_conv_s8_cuda_core_paths(cuda_lib, shape, groups, expect):
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st, dil = shape
    p = b2q.Conv2DParams(pad, pad, st, st, dil, dil, groups)
    paths = _conv_case(n, h, w, c, r, s, k, p, seed=7 + sum(shape), groups=groups)
    assert paths == set(expect.split("|")), paths


@pytest.mark.parametrize("shape", [
    # n, h, w, c, pad, stride
    (1, 112, 112, 32, 1, 1),    # two 56-column tiles per row block
    (2, 113, 111, 96, 1, 2),    # odd sizes, stride 2
    (1, 9, 300, 16, 1, 1),      # wide rows: three column tiles
    (3, 7, 7, 960, 1, 1),       # 4 channel slabs of 240
    (2, 14, 14, 576, 1, 2),     # 3 slabs of 192, stride 2
    (2, 5, 6, 144, 0, 1),       # no padding
    (1, 6, 9, 64, 2, 1),        # padding 2 (output larger than input)
    (5, 28, 28, 192, 1, 1),     # row groups: several threads per column
    (1, 3, 4, 16, 1, 2),        # tiny image
])
def test_depthwise_tma_int8(cuda_lib, shape):
    """TMA-staged depthwise 3x3 (int8 outputs): every clamp form against the oracle."""
    b2q = _b2q()
    n, h, w, c, pad, st = shape
    p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, c)
    x = rng_s8(sum(shape), (n, h, w, c))
    wt = rng_s8(sum(shape) + 1, (c, 3, 3, 1))
    rng = np.random.default_rng(sum(shape) + 2)
    bias = rng.integers(-2**15, 2**15 + 1, size=c).astype(np.int32)
    scale = rng.uniform(1e-3, 1e-2, size=c).astype(np.float32)
    acc = oracle.conv_s8(oracle.conv_args(n, h, w, c, 3, 3, c, pad, pad, st, st, 1, 1, c), x, wt, threads=4)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(wt).cuda()
    bd, sd = torch.from_numpy(bias).cuda(), torch.from_numpy(scale).cuda()
    for epi, (zp, lo, hi) in ((b2q.Epilogue.int8(), (0, -128, 127)), (b2q.Epilogue.int8(relu=True), (0, 0, 127)),
                              (b2q.Epilogue.int8(relu6_q=96), (0, 0, 96)), (b2q.Epilogue(1, 5, -100, 90), (5, -100, 90))):
        y = b2q.conv2d_s8(xd, wd, bd, sd, p, epi)
        torch.cuda.synchronize()
        assert b2q.last_path() == "cuda-core-depthwise-tma", b2q.last_path()
        np.testing.assert_array_equal(y.cpu().numpy(), oracle.requant_s8(acc, bias, scale, zp, lo, hi),
                                      err_msg=f"{shape} clamp {lo}..{hi} zp {zp}")


@pytest.mark.parametrize("shape", [
    (2, 56, 56, 24, 1, 1, 144, 0, 1, 1),   # MobileNetV2 expand 24 -> 144
    (2, 48, 48, 24, 3, 3, 40, 1, 1, 1),    # C = 24, 3x3, K = 40 (scalar edge stores)
])
def test_conv_s8_packed_low_channel(cuda_lib, shape):
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st, dil = shape
    p = b2q.Conv2DParams(pad, pad, st, st, dil, dil, 1)
    paths = _conv_case(n, h, w, c, r, s, k, p, seed=3 + sum(shape))
    assert paths == {"tcgen05-packed"}, paths


@pytest.mark.parametrize("shape", [
    # n, h, w, c, r, s, k, pad, stride, dil
    (4, 64, 64, 3, 7, 7, 64, 3, 2, 1),     # ResNet-50 stem geometry (7x7/2, C = 3): 4x4 tap pairs
    (2, 128, 128, 3, 3, 3, 32, 1, 2, 1),   # MobileNetV2 stem (3x3/2, C = 3 -> 32): 2x2 taps
    (3, 45, 39, 3, 7, 7, 64, 3, 2, 1),     # odd H / W: zero row / column in the last 2x2 blocks
    (3, 64, 64, 1, 3, 3, 16, 1, 2, 1),     # C = 1, N = 16
    (3, 40, 40, 4, 5, 5, 48, 2, 2, 1),     # C = 4, 5x5 pad 2: 3 x 4 taps, N = 48
    (3, 41, 41, 2, 3, 3, 40, 0, 2, 1),     # C = 2, no padding, N = 40 (scalar tail)
    (1, 40, 250, 3, 7, 7, 64, 3, 2, 1),    # Wo = 125: row pitch 128, one output row per tile
    (4, 32, 32, 3, 7, 7, 256, 3, 2, 1),    # N = 256
])
def test_conv_s8_tcgen05_s2d_stem(cuda_lib, shape):
    """Stride-2 low-channel convs (network stems; at least 1024 output pixels) as row tiles over a
    space-to-depth copy of the input: 2x2 pixel blocks become 16-channel pixels and each MMA slice
    covers two taps."""
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st, dil = shape
    p = b2q.Conv2DParams(pad, pad, st, st, dil, dil, 1)
    paths = _conv_case(n, h, w, c, r, s, k, p, seed=11 + sum(shape))
    assert paths == {"tcgen05-s2d"}, paths


@pytest.mark.parametrize("shape", [
    # n, h, w, c, r, s, k, pad, stride, dil
    (1, 56, 56, 64, 3, 3, 64, 1, 1, 1),
    (4, 56, 56, 64, 3, 3, 64, 1, 1, 1),    # ResNet-50 stage-1 3x3 (2 output rows per tile)
    (2, 13, 11, 64, 3, 3, 48, 1, 1, 1),    # ragged: H not a multiple of the tile rows, N = 48
    (3, 9, 127, 32, 3, 3, 32, 1, 1, 1),    # widest row (W + 1 = 128: one output row per tile)
    (2, 14, 14, 128, 3, 3, 64, 1, 1, 1),   # C = 128 (8 channel chunks per window)
    (2, 28, 28, 128, 3, 3, 128, 1, 1, 1),  # ResNet stage-2 3x3: 144 KiB of resident weights, 2 stages
    (2, 7, 5, 64, 3, 3, 40, 1, 1, 1),      # N = 40 (scalar tail), tiny image
    (1, 6, 6, 64, 3, 3, 64, 1, 1, 1),      # 36 output pixels: one tile, 6 rows
    (20, 56, 56, 64, 3, 3, 64, 1, 1, 1),   # 3 row groups per tile (4 would leave SMs idle): 384 -> 512 TMEM columns
    (12, 56, 56, 64, 3, 3, 64, 1, 1, 1),   # 2 row groups per tile
])
def test_conv_s8_tcgen05_rowtile(cuda_lib, shape):
    """3x3 stride-1 convs on row tiles (one window load per tile for all nine taps)."""
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st, dil = shape
    p = b2q.Conv2DParams(pad, pad, st, st, dil, dil, 1)
    paths = _conv_case(n, h, w, c, r, s, k, p, seed=sum(shape))
    assert paths == {"tcgen05-rowtile"}, paths


def test_conv_forced_cuda_core_matches_tcgen05(cuda_lib):
    b2q = _b2q()
    x = torch.from_numpy(rng_s8(5, (2, 32, 32, 64))).cuda()
    w = torch.from_numpy(rng_s8(6, (64, 3, 3, 64))).cuda()
    p = b2q.Conv2DParams()
    y_tc = b2q.conv2d_s8(x, w, None, None, p, b2q.Epilogue.int32())
    assert b2q.last_path() == "tcgen05-rowtile"
    b2q.set_path_policy(1)
    try:
        y_cc = b2q.conv2d_s8(x, w, None, None, p, b2q.Epilogue.int32())
        assert b2q.last_path() == "cuda-core-generic"
    finally:
        b2q.set_path_policy(0)
    torch.cuda.synchronize()
    assert torch.equal(y_tc, y_cc)


def test_conv_output_guard_band(cuda_lib):
    """Nothing is written past the output tensor (4 KiB poisoned tail)."""
    b2q = _b2q()
    n, h, w, c, k = 1, 48, 48, 64, 48
    x = torch.from_numpy(rng_s8(9, (n, h, w, c))).cuda()
    wt = torch.from_numpy(rng_s8(10, (k, 3, 3, c))).cuda()
    scale = torch.full((k,), 1e-3, device="cuda")
    numel = n * h * w * k
    buf = torch.full((numel + 4096,), 0x5A, dtype=torch.int8, device="cuda")
    b2q.conv2d_s8_into(buf, x, wt, None, scale, n, h, w, c, 3, 3, k, b2q.Conv2DParams(), b2q.Epilogue.int8())
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-rowtile"
    assert torch.all(buf[numel:] == 0x5A)


# ------------------------------------------------------------------ int8 bmm

@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_bmm_s8_tcgen05_transposes(cuda_lib, ta, tb):
    b2q = _b2q()
    batch, M, N, K = 3, 256, 384, 320
    A = rng_s8(20 + ta, (batch, K, M) if ta else (batch, M, K))
    B = rng_s8(30 + tb, (batch, N, K) if tb else (batch, K, N))
    acc = oracle.bmm_s8(A, B, batch, M, N, K, ta, tb, threads=4)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = b2q.bmm_s8(Ad, Bd, ta, tb, b2q.Epilogue.int32())
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-tiled"
    np.testing.assert_array_equal(C.cpu().numpy(), acc)
    scale = np.random.default_rng(3).uniform(1e-4, 1e-3, size=N).astype(np.float32)
    C8 = b2q.bmm_s8(Ad, Bd, ta, tb, b2q.Epilogue.int8(), col_scale=torch.from_numpy(scale).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(C8.cpu().numpy(), oracle.requant_s8(acc, None, scale))


@pytest.mark.parametrize("dims", [(1, 1, 1, 1), (2, 17, 19, 13), (2, 100, 36, 48), (1, 130, 64, 200)])
def test_bmm_s8_edges(cuda_lib, dims):
    b2q = _b2q()
    batch, M, N, K = dims
    for ta in (0, 1):
        for tb in (0, 1):
            A = rng_s8(M + ta, (batch, K, M) if ta else (batch, M, K))
            B = rng_s8(N + tb, (batch, N, K) if tb else (batch, K, N))
            C = b2q.bmm_s8(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), ta, tb, b2q.Epilogue.int32())
            torch.cuda.synchronize()
            np.testing.assert_array_equal(C.cpu().numpy(), oracle.bmm_s8(A, B, batch, M, N, K, ta, tb), err_msg=str((ta, tb)))


# ------------------------------------------------------------------ full-size properties

def test_config2_bmm_full_size_sampled(cuda_lib):
    """BASELINE config 2 at full size (64 x 1024^3, NN): tcgen05 == CUDA-core path bit for bit,
    and sampled rows equal an int64 numpy product."""
    b2q = _b2q()
    from my_own_cnn_b200 import synth

    batch, M, N, K = 64, 1024, 1024, 1024
    A = synth.fill_s8_uniform(torch.empty((batch, M, K), dtype=torch.int8, device="cuda"), 42, 101)
    B = synth.fill_s8_uniform(torch.empty((batch, K, N), dtype=torch.int8, device="cuda"), 42, 102)
    C = b2q.bmm_s8(A, B, 0, 0, b2q.Epilogue.int32())
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    b2q.set_path_policy(1)
    try:
        C2 = b2q.bmm_s8(A, B, 0, 0, b2q.Epilogue.int32())
    finally:
        b2q.set_path_policy(0)
    torch.cuda.synchronize()
    assert torch.equal(C, C2)
    for b in (0, 31, 63):
        Ah = synth.s8_uniform_host(42, 101, -127, 127, b * M * K, M * K).reshape(M, K)
        Bh = synth.s8_uniform_host(42, 102, -127, 127, b * K * N, K * N).reshape(K, N)
        rows = [0, 511, 1023]
        np.testing.assert_array_equal(C[b, rows].cpu().numpy(), Ah[rows].astype(np.int64) @ Bh.astype(np.int64))


def test_config4_pointwise_full_batch_sampled_images(cuda_lib):
    """BASELINE config 4a at full size (b512, 14x14, 1024->2048): sampled images vs the oracle."""
    b2q = _b2q()
    from my_own_cnn_b200 import synth

    n, h, w, c, k = 512, 14, 14, 1024, 2048
    x = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device="cuda"), 42, 401)
    wt = synth.fill_s8_uniform(torch.empty((k, 1, 1, c), dtype=torch.int8, device="cuda"), 42, 402)
    bias = synth.fill_i32_uniform(torch.empty(k, dtype=torch.int32, device="cuda"), 42, 403, -2**15, 2**15)
    scale_h = synth.scales_f32(k, 42, 404)
    y = b2q.conv2d_s8(x, wt, bias, torch.from_numpy(scale_h).cuda(), b2q.Conv2DParams(0, 0), b2q.Epilogue.int8())
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-tiled"
    wh = synth.s8_uniform_host(42, 402, -127, 127, 0, k * c).reshape(k, 1, 1, c)
    bh = synth.i32_uniform_host(42, 403, -2**15, 2**15, 0, k)
    for img in (0, 257, 511):
        xh = synth.s8_uniform_host(42, 401, -127, 127, img * h * w * c, h * w * c).reshape(1, h, w, c)
        acc = oracle.conv_s8(oracle.conv_args(1, h, w, c, 1, 1, k, 0, 0), xh, wh)
        np.testing.assert_array_equal(y[img:img + 1].cpu().numpy(), oracle.requant_s8(acc, bh, scale_h))


def test_pair_tiles_exact_on_long_reduction(cuda_lib):
    """2-SM tiles (cluster of two CTAs, M = 256 MMAs): config 4b geometry with a batch whose row
    count is not a multiple of 256; int32 accumulators compared in full with an exact float64
    product, int8 outputs of sampled images with the oracle."""
    b2q = _b2q()
    from my_own_cnn_b200 import synth

    n, h, w, c, k = 100, 14, 14, 2048, 512
    x = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device="cuda"), 42, 411)
    wt = synth.fill_s8_uniform(torch.empty((k, 1, 1, c), dtype=torch.int8, device="cuda"), 42, 412)
    acc = b2q.conv2d_s8(x, wt, None, None, b2q.Conv2DParams(0, 0), b2q.Epilogue.int32())
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    ref = (x.reshape(-1, c).double() @ wt.reshape(k, c).double().T).to(torch.int64)
    assert torch.equal(acc.reshape(-1, k).to(torch.int64), ref)
    bias = synth.fill_i32_uniform(torch.empty(k, dtype=torch.int32, device="cuda"), 42, 413, -2**15, 2**15)
    scale_h = synth.scales_f32(k, 42, 414)
    y = b2q.conv2d_s8(x, wt, bias, torch.from_numpy(scale_h).cuda(), b2q.Conv2DParams(0, 0), b2q.Epilogue.int8())
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    wh = synth.s8_uniform_host(42, 412, -127, 127, 0, k * c).reshape(k, 1, 1, c)
    bh = synth.i32_uniform_host(42, 413, -2**15, 2**15, 0, k)
    for img in (0, 51, 99):
        xh = synth.s8_uniform_host(42, 411, -127, 127, img * h * w * c, h * w * c).reshape(1, h, w, c)
        a = oracle.conv_s8(oracle.conv_args(1, h, w, c, 1, 1, k, 0, 0), xh, wh)
        np.testing.assert_array_equal(y[img:img + 1].cpu().numpy(), oracle.requant_s8(a, bh, scale_h))


# ------------------------------------------------------------------ failure path

def test_bounded_wait_timeout_reports_and_context_survives(cuda_lib):
    b2q = _b2q()
    from my_own_cnn_b200 import _lib

    rc = _lib.lib().b200q_selftest_wait_timeout(20000)
    assert rc == _lib.B200Q_ERR_TIMEOUT
    assert b"wait ran out" in _lib.lib().b200q_last_error()
    assert _lib.lib().b200q_device_error() == 0  # cleared
    # the context is still usable
    x = torch.from_numpy(rng_s8(1, (1, 8, 8, 64))).cuda()
    w = torch.from_numpy(rng_s8(2, (16, 1, 1, 64))).cuda()
    y = b2q.conv2d_s8(x, w, None, None, b2q.Conv2DParams(0, 0), b2q.Epilogue.int32())
    torch.cuda.synchronize()
    assert y.shape == (1, 8, 8, 16)


def test_no_device_error_after_suite(cuda_lib):
    from my_own_cnn_b200 import _lib

    assert _lib.lib().b200q_device_error() == 0, _lib.lib().b200q_last_error()


def test_conv_stack_pipelined_host_pass_matches_oracle(cuda_lib):
    """ConvStack.run_host (chunked H2D / kernels / D2H on three streams, ragged last chunk)
    equals the device-resident pass and the oracle."""
    b2q = _b2q()
    from my_own_cnn_b200.stack import ConvLayer, ConvStack

    n, h, w, c, k1, k2 = 37, 20, 20, 64, 96, 32
    x = rng_s8(50, (n, h, w, c))
    w1, w2 = rng_s8(51, (k1, 3, 3, c)), rng_s8(52, (k2, 1, 1, k1))
    rng = np.random.default_rng(53)
    b1 = rng.integers(-2**15, 2**15, size=k1).astype(np.int32)
    s1 = rng.uniform(1e-4, 1e-3, size=k1).astype(np.float32)
    s2 = rng.uniform(1e-3, 1e-2, size=k2).astype(np.float32)
    cu = lambda a: torch.from_numpy(a).cuda()
    net = ConvStack([ConvLayer(cu(w1), cu(b1), cu(s1), b2q.Conv2DParams(), b2q.Epilogue.int8(relu=True)),
                     ConvLayer(cu(w2), None, cu(s2), b2q.Conv2DParams(0, 0), b2q.Epilogue.int32())], (h, w, c))
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((n, h, w, k2), dtype=torch.int32).pin_memory()
    net.run_host(xh, yh, chunk=8)
    torch.cuda.synchronize()
    y_dev = net.forward(cu(x)).cpu()
    acc1 = oracle.conv_s8(oracle.conv_args(n, h, w, c, 3, 3, k1), x, w1, threads=4)
    y1 = oracle.requant_s8(acc1, b1, s1, 0, 0, 127)
    ref = oracle.conv_s8(oracle.conv_args(n, h, w, k1, 1, 1, k2, 0, 0), y1, w2, threads=4)
    np.testing.assert_array_equal(yh.numpy(), ref)
    np.testing.assert_array_equal(y_dev.numpy(), ref)


def test_matches_reference_gpu_implementation(cuda_lib):
    """The reference's own CUDA quantized conv (compiled unmodified into oracle/_ref/libref_gpu.so)
    and this library give identical int32 accumulators, on the tensor-core and CUDA-core paths."""
    import ctypes

    b2q = _b2q()
    lib = ROOT / "oracle" / "_ref" / "libref_gpu.so"
    if not lib.exists():
        pytest.skip("reference GPU library not built (needs the reference sources at build time)")
    ref = ctypes.CDLL(str(lib))
    ref.refgpu_fprop_qi32_s5.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 9 + [ctypes.c_void_p] * 2
    for (n, h, w, c, r, k, pad, st) in [(2, 40, 40, 64, 3, 96, 1, 1), (3, 14, 14, 256, 1, 128, 0, 1),
                                        (2, 23, 23, 3, 7, 64, 3, 2), (1, 9, 9, 24, 3, 8, 1, 2)]:
        x8 = torch.from_numpy(rng_s8(n + c, (n, h, w, c))).cuda()
        w8 = torch.from_numpy(rng_s8(k + r, (k, r, r, c))).cuda()
        p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, 1)
        ho, wo = b2q.conv_out_shape(h, w, c, r, r, k, p)
        y_ref = torch.zeros((n, ho, wo, k), dtype=torch.int32, device="cuda")
        qp_in = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)] * n)
        qp_f = b2q.qparams_to_device([b2q.QuantizationParametersS5(0, 31, 1.0)])
        xf, wf = x8.float(), w8.float()
        assert ref.refgpu_fprop_qi32_s5(xf.data_ptr(), wf.data_ptr(), y_ref.data_ptr(), n, h, w, c, r, r, k, pad, st,
                                        qp_in.data_ptr(), qp_f.data_ptr()) == 0
        y = b2q.conv2d_s8(x8, w8, None, None, p, b2q.Epilogue.int32())
        torch.cuda.synchronize()
        assert torch.equal(y, y_ref), (n, h, w, c, r, k)


@pytest.mark.parametrize("args", [
    ["--op", "all", "--qtype", "u8"],                                             # BASELINE config 1 shape
    ["--op", "qfprop", "--qtype", "s5", "--custom_mode", "blocked", "--n", "4", "--block_by", "2", "--block_bx", "2"],
    ["--op", "all", "--qtype", "u8", "--n", "2", "--h", "28", "--w", "28", "--c", "64", "--k", "64", "--groups", "4"],
    ["--op", "all", "--qtype", "s5", "--n", "3", "--h", "14", "--w", "14", "--c", "256", "--k", "512", "--r", "1",
     "--s", "1", "--pad_h", "0", "--pad_w", "0"],
])
def test_cpp_qconv_bench_driver(cuda_lib, args):
    """The C++ driver (shim/qconv_bench.cu: the reference's conv_bench pattern, benchmark_cuda_op from the
    reference's src/bench.cpp) calls the reference's quantized entry points and the int8 C ABI, and its
    exact check against the reference's cpu_ref.cpp passes."""
    binary = ROOT / "oracle" / "_ref" / "qconv_bench_b200"
    if not binary.exists():
        pytest.skip("qconv_bench not built (needs the reference sources at build time)")
    proc = subprocess.run([str(binary), *args, "--warmup", "2", "--iters", "5", "--check"], capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "qconv_bench PASS" in proc.stdout, proc.stdout
    assert "custom qfprop" in proc.stdout or "custom s8" in proc.stdout
    assert "gflops=" in proc.stdout
    if "qfprop" in args or "all" in args:
        assert "path 11" in proc.stdout, proc.stdout  # the drop-in ran on the tcgen05 route


@pytest.mark.parametrize("shape", [
    # n, h, w, c, r, k, pad: GEMMs of >= 2^36 MACs with 128-byte K blocks (prepacked weights)
    (300, 14, 14, 1088, 1, 1024, 0),  # 1x1 tiled, C = 8.5 x 128 (last K block half zero)
    (16, 56, 56, 320, 3, 512, 1),     # 3x3 im2col, C = 2.5 x 128 per tap
])
def test_prepacked_weights_long_reduction(cuda_lib, shape):
    """Long-reduction convs whose weights go through the per-stage prepack (one bulk copy per
    stage): int32 accumulators and int8 outputs of sampled images against the oracle."""
    b2q = _b2q()
    n, h, w, c, r, k, pad = shape
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = torch.randint(-128, 128, (n, h, w, c), dtype=torch.int8, device="cuda", generator=g)
    wt = torch.randint(-128, 128, (k, r, r, c), dtype=torch.int8, device="cuda", generator=g)
    bias = torch.randint(-2**15, 2**15, (k,), dtype=torch.int32, device="cuda", generator=g)
    scale = torch.rand(k, device="cuda", generator=g) * 1e-5 + 1e-6
    p = b2q.Conv2DParams(pad, pad, 1, 1, 1, 1, 1)
    y32 = b2q.conv2d_s8(x, wt, None, None, p, b2q.Epilogue.int32())
    y8 = b2q.conv2d_s8(x, wt, bias, scale, p, b2q.Epilogue.int8(relu=True))
    torch.cuda.synchronize()
    assert b2q.last_path() == ("tcgen05-tiled" if r == 1 else "tcgen05-im2col")
    wh, bh, sh = wt.cpu().numpy(), bias.cpu().numpy(), scale.cpu().numpy()
    for img in (0, n // 2, n - 1):
        xh = x[img:img + 1].cpu().numpy()
        acc = oracle.conv_s8(oracle.conv_args(1, h, w, c, r, r, k, pad, pad), xh, wh, threads=8)
        np.testing.assert_array_equal(y32[img:img + 1].cpu().numpy(), acc)
        np.testing.assert_array_equal(y8[img:img + 1].cpu().numpy(), oracle.requant_s8(acc, bh, sh, 0, 0, 127))


@pytest.mark.parametrize("tb", [0, 1])
def test_bmm_s8_2sm_tiles_both_b_layouts(cuda_lib, tb):
    """bmm on 2-SM tiles with B stored [K][N] (MN-major operand) or [N][K] (K-major): every
    int32 output against an exact product, int8 outputs against the oracle's requantization."""
    b2q = _b2q()
    batch, M, N, K = 40, 512, 768, 384
    g = torch.Generator(device="cuda").manual_seed(77 + tb)
    A = torch.randint(-128, 128, (batch, M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-128, 128, (batch, N, K) if tb else (batch, K, N), dtype=torch.int8, device="cuda", generator=g)
    bias = torch.randint(-2**15, 2**15, (N,), dtype=torch.int32, device="cuda", generator=g)
    scale = torch.rand(N, device="cuda", generator=g) * 1e-4 + 1e-6
    C32 = b2q.bmm_s8(A, B, 0, tb, b2q.Epilogue.int32())
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    C8 = b2q.bmm_s8(A, B, 0, tb, b2q.Epilogue.int8(), bias=bias, col_scale=scale)
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    torch.cuda.synchronize()
    Ah = A.cpu().numpy().astype(np.float64)
    Bh = B.cpu().numpy().astype(np.float64)
    want = np.matmul(Ah, np.swapaxes(Bh, 1, 2) if tb else Bh).astype(np.int64).astype(np.int32)
    np.testing.assert_array_equal(C32.cpu().numpy(), want)
    np.testing.assert_array_equal(C8.cpu().numpy(), oracle.requant_s8(want, bias.cpu().numpy(), scale.cpu().numpy()))
