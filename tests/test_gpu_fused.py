"""GPU parity of the widened int8 network pieces: the residual add fused into the conv epilogue
(every conv path), int8 max / global-average pooling, and a ResNet-50 bottleneck block chained on
the device.  Bar: bit-exact against the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.kat import rng_s8

pytestmark = pytest.mark.gpu
RES_SCALE = 0.43


def _b2q():
    import my_own_cnn_b200 as b2q

    return b2q


@pytest.mark.parametrize("shape,expect", [
    ((8, 28, 28, 64, 1, 1, 256, 0, 1), "tcgen05-tiled"),      # reduction 64 < 128: direct 16-byte stores
    ((4, 14, 14, 256, 1, 1, 512, 0, 1), "tcgen05-tiled"),     # reduction 256: TMA-store epilogue
    ((4, 28, 28, 64, 3, 3, 64, 1, 1), "tcgen05-rowtile"),
    ((4, 28, 28, 128, 3, 3, 128, 1, 1), "tcgen05-rowtile"),   # 144 KiB of resident weights
    ((4, 14, 14, 256, 3, 3, 256, 1, 1), "tcgen05-im2col"),
    ((4, 64, 64, 3, 7, 7, 64, 3, 2), "tcgen05-s2d"),           # C = 3 stem geometry
    ((2, 56, 56, 24, 3, 3, 40, 1, 1), "tcgen05-packed"),       # C = 24: im2col pack
    ((1, 6, 6, 48, 3, 3, 64, 1, 1), "cuda-core-generic"),
    ((3, 7, 9, 32, 1, 1, 48, 0, 1), "tcgen05-tiled"),         # ragged M, N = 48 (16-column tail)
])
def test_conv_residual_add_matches_oracle(cuda_lib, shape, expect):
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st = shape
    p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, 1)
    seed = 500 + sum(shape)
    x, wt = rng_s8(seed, (n, h, w, c)), rng_s8(seed + 1, (k, r, s, c))
    rng = np.random.default_rng(seed + 2)
    bias = rng.integers(-2**15, 2**15 + 1, size=k).astype(np.int32)
    scale = rng.uniform(1e-4, 1e-3, size=k).astype(np.float32)
    ho, wo = b2q.conv_out_shape(h, w, c, r, s, k, p)
    res = rng_s8(seed + 3, (n, ho, wo, k), -128, 127)
    acc = oracle.conv_s8(oracle.conv_args(n, h, w, c, r, s, k, pad, pad, st, st), x, wt, threads=4)
    d = lambda a: torch.from_numpy(a).cuda()
    for lo, hi, epi in [(-128, 127, b2q.Epilogue.int8()), (0, 127, b2q.Epilogue.int8(relu=True))]:
        y = b2q.conv2d_s8_add(d(x), d(wt), d(bias), d(scale), d(res), RES_SCALE, p, epi)
        torch.cuda.synchronize()
        assert b2q.last_path() == expect
        want = oracle.requant_res_s8(acc, bias, scale, res, RES_SCALE, 0, lo, hi)
        np.testing.assert_array_equal(y.cpu().numpy(), want)


def test_conv_residual_add_on_2sm_tiles(cuda_lib):
    """Long reduction (2-SM tiles): int32 accumulators from the device (exact, checked elsewhere)
    requantized with the residual by the oracle, against the fused device result."""
    b2q = _b2q()
    from my_own_cnn_b200 import synth

    n, h, w, c, k = 100, 14, 14, 2048, 512
    p = b2q.Conv2DParams(0, 0)
    x = synth.fill_s8_uniform(torch.empty((n, h, w, c), dtype=torch.int8, device="cuda"), 9, 1)
    wt = synth.fill_s8_uniform(torch.empty((k, 1, 1, c), dtype=torch.int8, device="cuda"), 9, 2)
    res = synth.fill_s8_uniform(torch.empty((n, h, w, k), dtype=torch.int8, device="cuda"), 9, 3, -128, 127)
    bias = synth.fill_i32_uniform(torch.empty(k, dtype=torch.int32, device="cuda"), 9, 4, -2**15, 2**15)
    scale = torch.from_numpy(synth.scales_f32(k, 9, 5)).cuda()
    acc = b2q.conv2d_s8(x, wt, None, None, p, b2q.Epilogue.int32())
    y = b2q.conv2d_s8_add(x, wt, bias, scale, res, RES_SCALE, p, b2q.Epilogue.int8(relu=True))
    torch.cuda.synchronize()
    assert b2q.last_path() == "tcgen05-tiled-2sm"
    want = oracle.requant_res_s8(acc.cpu().numpy(), bias.cpu().numpy(), scale.cpu().numpy(), res.cpu().numpy(),
                                 RES_SCALE, 0, 0, 127)
    np.testing.assert_array_equal(y.cpu().numpy(), want)


def test_conv_residual_add_rejects_bad_arguments(cuda_lib):
    b2q = _b2q()
    x = torch.zeros((1, 8, 8, 32), dtype=torch.int8, device="cuda")
    wt = torch.zeros((32, 1, 1, 32), dtype=torch.int8, device="cuda")
    sc = torch.ones(32, device="cuda")
    with pytest.raises(RuntimeError, match="residual shape"):
        b2q.conv2d_s8_add(x, wt, None, sc, torch.zeros((1, 8, 8, 16), dtype=torch.int8, device="cuda"), 1.0,
                          b2q.Conv2DParams(0, 0), b2q.Epilogue.int8())
    y = torch.empty((1, 8, 8, 32), dtype=torch.int32, device="cuda")
    with pytest.raises(b2q.B200QError, match="int8 outputs"):
        b2q.conv2d_s8_add_into(y, x, wt, None, sc, x, 1.0, 1, 8, 8, 32, 1, 1, 32, b2q.Conv2DParams(0, 0),
                               b2q.Epilogue.int32())


@pytest.mark.parametrize("shape,win", [
    ((2, 112, 112, 64), (3, 2, 1)),    # ResNet-50 max pool
    ((3, 9, 11, 24), (3, 2, 1)),       # C % 16 != 0: per-element kernel
    ((1, 8, 8, 32), (2, 2, 0)),
    ((2, 5, 7, 16), (3, 1, 1)),
])
def test_maxpool_matches_oracle(cuda_lib, shape, win):
    b2q = _b2q()
    r, st, pad = win
    x = rng_s8(700 + sum(shape), shape, -128, 127)
    y = b2q.maxpool_s8(torch.from_numpy(x).cuda(), r, r, st, pad)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.maxpool_s8(x, r, r, st, st, pad, pad))


@pytest.mark.parametrize("shape", [(4, 7, 7, 2048), (2, 5, 3, 40), (1, 1, 1, 8)])
def test_global_avgpool_matches_oracle(cuda_lib, shape):
    b2q = _b2q()
    x = rng_s8(800 + sum(shape), shape, -128, 127)
    y = b2q.global_avgpool_s8(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), oracle.global_avgpool_s8(x))


def test_resnet_bottleneck_block_chained_on_device(cuda_lib):
    """conv1 1x1 -> conv2 3x3 -> conv3 1x1 + shortcut (ReLU epilogues), the stage-1 block of
    ResNet-50 at batch 2, every intermediate int8 tensor staying on the device."""
    b2q = _b2q()
    n, hw, cin, width = 2, 56, 256, 64
    rng = np.random.default_rng(900)
    x = rng_s8(901, (n, hw, hw, cin), 0, 127)
    ws = [rng_s8(902, (width, 1, 1, cin)), rng_s8(903, (width, 3, 3, width)), rng_s8(904, (cin, 1, 1, width))]
    bs = [rng.integers(-2**15, 2**15, size=wt.shape[0]).astype(np.int32) for wt in ws]
    ss = [rng.uniform(1e-4, 1e-3, size=wt.shape[0]).astype(np.float32) for wt in ws]
    d = lambda a: torch.from_numpy(a).cuda()
    relu = b2q.Epilogue.int8(relu=True)
    y1 = b2q.conv2d_s8(d(x), d(ws[0]), d(bs[0]), d(ss[0]), b2q.Conv2DParams(0, 0), relu)
    y2 = b2q.conv2d_s8(y1, d(ws[1]), d(bs[1]), d(ss[1]), b2q.Conv2DParams(1, 1), relu)
    y3 = b2q.conv2d_s8_add(y2, d(ws[2]), d(bs[2]), d(ss[2]), d(x), RES_SCALE, b2q.Conv2DParams(0, 0), relu)
    torch.cuda.synchronize()
    a1 = oracle.requant_s8(oracle.conv_s8(oracle.conv_args(n, hw, hw, cin, 1, 1, width, 0, 0), x, ws[0], 4),
                           bs[0], ss[0], 0, 0, 127)
    a2 = oracle.requant_s8(oracle.conv_s8(oracle.conv_args(n, hw, hw, width, 3, 3, width), a1, ws[1], 4),
                           bs[1], ss[1], 0, 0, 127)
    a3 = oracle.requant_res_s8(oracle.conv_s8(oracle.conv_args(n, hw, hw, width, 1, 1, cin, 0, 0), a2, ws[2], 4),
                               bs[2], ss[2], x, RES_SCALE, 0, 0, 127)
    np.testing.assert_array_equal(y3.cpu().numpy(), a3)


@pytest.mark.parametrize("shape,expect", [
    ((8, 28, 28, 64, 1, 1, 256, 0, 1), "tcgen05-tiled"),      # direct 16-byte stores
    ((4, 14, 14, 256, 1, 1, 512, 0, 1), "tcgen05-tiled"),     # TMA-store epilogue
    ((4, 28, 28, 64, 3, 3, 64, 1, 1), "tcgen05-rowtile"),
    ((3, 7, 9, 32, 1, 1, 48, 0, 1), "tcgen05-tiled"),         # 16-column tail
    ((2, 28, 28, 144, 1, 1, 24, 0, 1), "tcgen05-tiled"),      # N = 24: 8-byte rows (MobileNetV2 project)
    ((3, 7, 9, 32, 1, 1, 40, 0, 1), "tcgen05-tiled"),         # N = 40: 32 + 8-column tail, 8-byte rows
])
@pytest.mark.parametrize("with_res", [False, True])
def test_clamp_forms_with_special_scales(cuda_lib, shape, expect, with_res):
    """Every clamp form of the int8 epilogue (default range, ReLU / ReLU6 clamped in floats before
    the conversion, general bounds with a zero point) against the oracle, with per-column scales
    that include NaN, +-inf, zero, negative and huge values and large biases: NaN products must
    become 0 before the clamp, infinities saturate."""
    b2q = _b2q()
    n, h, w, c, r, s, k, pad, st = shape
    p = b2q.Conv2DParams(pad, pad, st, st, 1, 1, 1)
    seed = 900 + sum(shape)
    x, wt = rng_s8(seed, (n, h, w, c)), rng_s8(seed + 1, (k, r, s, c))
    rng = np.random.default_rng(seed + 2)
    bias = rng.integers(-2**31, 2**31, size=k, dtype=np.int64).astype(np.int32)
    bias[: k // 2] = rng.integers(-2**12, 2**12, size=k // 2)
    scale = rng.uniform(-2e-3, 2e-3, size=k).astype(np.float32)
    special = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 3e38, -3e38, 1e-30, 0.5, -7.0], dtype=np.float32)
    scale[: len(special)] = special
    ho, wo = b2q.conv_out_shape(h, w, c, r, s, k, p)
    res = rng_s8(seed + 3, (n, ho, wo, k), -128, 127)
    acc = oracle.conv_s8(oracle.conv_args(n, h, w, c, r, s, k, pad, pad, st, st), x, wt, threads=4)
    d = lambda a: torch.from_numpy(a).cuda()
    forms = [(b2q.Epilogue.int8(), 0, -128, 127), (b2q.Epilogue.int8(relu=True), 0, 0, 127),
             (b2q.Epilogue.int8(relu6_q=96), 0, 0, 96), (b2q.Epilogue.int8(relu=True, zp_out=-5), -5, -5, 127),
             (b2q.Epilogue(1, 3, -100, 90), 3, -100, 90)]
    for epi, zp, lo, hi in forms:
        if with_res:
            y = b2q.conv2d_s8_add(d(x), d(wt), d(bias), d(scale), d(res), RES_SCALE, p, epi)
            want = oracle.requant_res_s8(acc, bias, scale, res, RES_SCALE, zp, lo, hi)
        else:
            y = b2q.conv2d_s8(d(x), d(wt), d(bias), d(scale), p, epi)
            want = oracle.requant_s8(acc, bias, scale, zp, lo, hi)
        torch.cuda.synchronize()
        assert b2q.last_path() == expect
        np.testing.assert_array_equal(y.cpu().numpy(), want, err_msg=f"zp={zp} lo={lo} hi={hi}")
