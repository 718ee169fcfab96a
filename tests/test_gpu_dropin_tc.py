"""The reference's own quantized-int32 entry points on the tensor-core route.

launch_fprop_nhwc_qi32 / launch_block_fprop_nhwc_qi32 (src/conv_types.h:232-251) take float codes
with per-image input zero points and one filter zero point.  Their tensor-core route packs the raw
codes as 8-bit operands (U8 unsigned, S5 signed) and restores the zero points with per-row and
per-column correction terms; codes that do not fit 8 bits fall back to a direct computation on the
device.  Every result here must equal the reference's own CPU code (src/cpu_ref.cpp, compiled
from its sources into oracle/_ref) bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.golden.make_golden import codes, filter_zp, input_zps
from tests.kat import kat_cases

pytestmark = pytest.mark.gpu
U8, S5 = 0, 1


def _b2q():
    import my_own_cnn_b200 as b2q

    return b2q


def _qp(kind, zps):
    b2q = _b2q()
    if kind == U8:
        return b2q.qparams_to_device([b2q.QuantizationParametersU8(int(z) & 0xFF, 0.25) for z in zps])
    return b2q.qparams_to_device([b2q.QuantizationParametersS5(int(z), 31, 0.5) for z in zps])


def _run(kind, x, wt, n, h, w, c, r, s, k, prm, blk=None, zin=None, zf=None):
    """Drop-in call through the C ABI; returns (y, path)."""
    b2q = _b2q()
    zin = input_zps(kind, n) if zin is None else zin
    zf = filter_zp(kind) if zf is None else zf
    p = b2q.Conv2DParams(*prm)
    ho, wo = b2q.conv_out_shape(h, w, c, r, s, k, p)
    y = torch.full((n, ho, wo, k), 0x7EADBEEF, dtype=torch.int32, device="cuda")
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32).reshape(-1)).cuda()
    wd = torch.from_numpy(np.ascontiguousarray(wt, dtype=np.float32).reshape(-1)).cuda()
    qt = b2q.DataType.LinQuantU8 if kind == U8 else b2q.DataType.LinQuantS5
    if blk:
        b2q.launch_block_fprop_nhwc_qi32(xd, wd, y, n, h, w, c, r, s, k, b2q.BlockConv2DParams(p, *blk),
                                         _qp(kind, zin), _qp(kind, [zf]), qtype=qt)
    else:
        b2q.launch_fprop_nhwc_qi32(xd, wd, y, n, h, w, c, r, s, k, p, _qp(kind, zin), _qp(kind, [zf]), qtype=qt)
    torch.cuda.synchronize()
    return y.cpu().numpy(), b2q.last_path()


def _ref(kind, x, wt, n, h, w, c, r, s, k, prm, blk=None, zin=None, zf=None):
    by, bx = blk or (1, 1)
    a = oracle.conv_args(n, h, w, c, r, s, k, *prm, by, bx)
    zin = input_zps(kind, n) if zin is None else zin
    zf = filter_zp(kind) if zf is None else zf
    return oracle.ref_conv_qi32(a, kind, x, wt, zin, zf, blk is not None)


def test_known_answers_on_both_datapaths(cuda_lib, golden):
    """The 12 golden cases: tensor-core route under automatic dispatch, CUDA-core kernel when forced."""
    b2q = _b2q()
    for policy, want in ((0, "tcgen05-qi32"), (1, "cuda-core-qi32")):
        b2q.set_path_policy(policy)
        try:
            for kc in kat_cases(golden):
                prm = (kc.pad_h, kc.pad_w, kc.stride_h, kc.stride_w, kc.dil_h, kc.dil_w, kc.groups)
                y, path = _run(kc.kind, kc.x, kc.wt, kc.n, kc.h, kc.w, kc.c, kc.r, kc.s, kc.k, prm,
                               (kc.by, kc.bx) if kc.blocked else None, kc.zp_in, kc.zp_f)
                np.testing.assert_array_equal(y, kc.y, err_msg=f"{kc.name} policy {policy}")
                tiny_groups = (kc.c // kc.groups) * (kc.k // kc.groups) <= 16  # direct kernel by design
                assert path == ("cuda-core-qi32" if tiny_groups else want), (kc.name, path)
        finally:
            b2q.set_path_policy(0)


@pytest.mark.parametrize("kind", [U8, S5])
def test_config1_shape_reference_zero_points(cuda_lib, kind):
    """BASELINE config 1 geometry (1x56x56x64, 3x3 pad 1, K = 64) with the reference test's code and
    zero-point formulas (quant_conv_test.cu:20-81): centred U8 values reach +-255."""
    n, h, w, c, r, s, k = 1, 56, 56, 64, 3, 3, 64
    prm = (1, 1, 1, 1, 1, 1, 1)
    x = codes(kind, n * h * w * c, 3).reshape(n, h, w, c)
    wt = codes(kind, k * r * s * c, 9)
    y, path = _run(kind, x, wt, n, h, w, c, r, s, k, prm)
    assert path == "tcgen05-qi32"
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm))


def test_batched_images_distinct_zero_points(cuda_lib):
    """Four images, each with its own zero point, stride 2 and a 5x5 filter of 24 channels."""
    kind = U8
    n, h, w, c, r, s, k = 4, 33, 29, 24, 5, 5, 40
    prm = (2, 2, 2, 2, 1, 1, 1)
    x = codes(kind, n * h * w * c, 5).reshape(n, h, w, c)
    wt = codes(kind, k * r * s * c, 2)
    zin = np.array([0, 255, 128, 17], dtype=np.int32)
    y, path = _run(kind, x, wt, n, h, w, c, r, s, k, prm, zin=zin, zf=200)
    assert path == "tcgen05-qi32"
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm, zin=zin, zf=200))


@pytest.mark.parametrize("kind", [U8, S5])
def test_blocked_realistic_shape(cuda_lib, kind):
    """Blocked conv at a realistic size: 4x56x56x64, 3x3, K = 64, 2x2 output blocks."""
    n, h, w, c, r, s, k = 4, 56, 56, 64, 3, 3, 64
    prm = (1, 1, 1, 1, 1, 1, 1)
    x = codes(kind, n * h * w * c, 1).reshape(n, h, w, c)
    wt = codes(kind, k * 2 * 2 * r * s * c, 4)
    y, path = _run(kind, x, wt, n, h, w, c, r, s, k, prm, blk=(2, 2))
    assert path == "tcgen05-qi32"
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm, blk=(2, 2)))


@pytest.mark.parametrize("groups", [2, 8, 32])
def test_grouped_and_depthwise(cuda_lib, groups):
    kind = S5
    n, h, w, c, r, s, k = 2, 20, 18, 32, 3, 3, 32
    prm = (1, 1, 1, 1, 1, 1, groups)
    x = codes(kind, n * h * w * c, 6).reshape(n, h, w, c)
    wt = codes(kind, k * r * s * (c // groups), 8)
    y, path = _run(kind, x, wt, n, h, w, c, r, s, k, prm)
    # groups of 4 x 4 channels or fewer run on the direct kernel (a GEMM per group would be 1-4 wide)
    assert path == ("cuda-core-qi32" if (c // groups) * (k // groups) <= 16 else "tcgen05-qi32")
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm))


def test_pointwise_config4_shape(cuda_lib):
    """Config 4a geometry (14x14, 1x1, C 1024 -> K 2048) on 2 images through the drop-in, zero points 0:
    equals the int8 conv's accumulators (itself checked against the oracle elsewhere) and sampled
    outputs of the reference CPU code."""
    b2q = _b2q()
    n, h, w, c, k = 2, 14, 14, 1024, 2048
    rng = np.random.default_rng(77)
    x8 = rng.integers(-127, 128, size=(n, h, w, c)).astype(np.int8)
    w8 = rng.integers(-127, 128, size=(k, 1, 1, c)).astype(np.int8)
    prm = (0, 0, 1, 1, 1, 1, 1)
    zin = np.zeros(n, dtype=np.int32)
    y, path = _run(S5, x8, w8, n, h, w, c, 1, 1, k, prm, zin=zin, zf=0)
    assert path == "tcgen05-qi32"
    y8 = b2q.conv2d_s8(torch.from_numpy(x8).cuda(), torch.from_numpy(w8).cuda(), None, None,
                       b2q.Conv2DParams(*prm), b2q.Epilogue.int32())
    np.testing.assert_array_equal(y, y8.cpu().numpy())
    ref = _ref(S5, x8[:1], w8, 1, h, w, c, 1, 1, k, prm, zin=zin[:1], zf=0)
    np.testing.assert_array_equal(y[:1], ref)


@pytest.mark.parametrize("kind", [U8, S5])
def test_codes_outside_8_bits_fall_back_on_device(cuda_lib, kind):
    """Codes that do not fit the 8-bit operand type (U8 below 0 or above 255, S5 beyond int8) are
    still exact: the device-side flag switches the correction pass to a direct computation."""
    n, h, w, c, r, s, k = 2, 9, 10, 8, 3, 3, 12
    prm = (1, 1, 1, 1, 1, 1, 1)
    x = codes(kind, n * h * w * c, 2).reshape(n, h, w, c).copy()
    wt = codes(kind, k * r * s * c, 3).copy()
    x[1, 4, 5, 3] = 300.0 if kind == U8 else 200.0
    wt[17] = -2.0 if kind == U8 else -150.0
    y, path = _run(kind, x, wt, n, h, w, c, r, s, k, prm)
    assert path == "tcgen05-qi32"
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm))
    # the next in-range call takes the tensor-core result again: the flag still holds the earlier
    # call's generation number, which this call's number does not match
    x[1, 4, 5, 3] = 7.0
    wt[17] = 5.0
    y, _ = _run(kind, x, wt, n, h, w, c, r, s, k, prm)
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm))


def test_fractional_codes_truncate(cuda_lib):
    """Float codes are cast with truncation, like static_cast<int32_t> (cpu_ref.cpp:15,23)."""
    kind = U8
    n, h, w, c, r, s, k = 1, 8, 8, 16, 3, 3, 16
    prm = (1, 1, 1, 1, 1, 1, 1)
    x = codes(kind, n * h * w * c, 1).reshape(n, h, w, c) + np.float32(0.75)
    wt = codes(kind, k * r * s * c, 2) + np.float32(0.5)
    y, _ = _run(kind, x, wt, n, h, w, c, r, s, k, prm)
    np.testing.assert_array_equal(y, _ref(kind, x, wt, n, h, w, c, r, s, k, prm))
