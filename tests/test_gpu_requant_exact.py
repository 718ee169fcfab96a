"""int8 requantization of short-reduction GEMMs (the epilogue-bound ones) against the CPU oracle.

Power-of-two scales put many products exactly on .5 (ties to even), every clamp form and zero
point is taken, the fused residual add with small and huge residual scales, large biases that wrap
the int32 sum, and NaN / inf / huge scales.  Bar: bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.kat import rng_s8

pytestmark = pytest.mark.gpu


def _b2q():
    import my_own_cnn_b200 as b2q

    return b2q


def _epilogues():
    b2q = _b2q()
    from my_own_cnn_b200 import _lib

    return [
        ("default", b2q.Epilogue.int8(), 0, -128, 127),
        ("relu", b2q.Epilogue.int8(relu=True), 0, 0, 127),
        ("relu6", b2q.Epilogue.int8(relu6_q=97), 0, 0, 97),
        ("zp", b2q.Epilogue(_lib.OUT_S8, 7, -100, 90), 7, -100, 90),
        ("zp_neg", b2q.Epilogue(_lib.OUT_S8, -3, -3, 127), -3, -3, 127),
    ]


def _scales(k, seed, special=None):
    rng = np.random.default_rng(seed)
    choices = np.array([2.0**-9, 2.0**-10, 2.0**-8, 0.5, 2.0**-12], dtype=np.float32)
    sc = np.where(rng.random(k) < 0.6, choices[rng.integers(0, len(choices), k)],
                  rng.uniform(1e-4, 4e-3, k)).astype(np.float32)
    if special is not None:
        for i, v in special.items():
            sc[i] = v
    return sc


def _case(n, h, w, c, r, k, pad, stride, bias_hi, special=None, res_scale=None, seed=0):
    b2q = _b2q()
    x = rng_s8(seed, (n, h, w, c), -128, 127)
    wt = rng_s8(seed + 1, (k, r, r, c), -128, 127)
    rng = np.random.default_rng(seed + 2)
    bias = rng.integers(-bias_hi, bias_hi + 1, size=k).astype(np.int32)
    scale = _scales(k, seed + 3, special)
    p = b2q.Conv2DParams(pad, pad, stride, stride, 1, 1, 1)
    acc = oracle.conv_s8(oracle.conv_args(n, h, w, c, r, r, k, pad, pad, stride, stride, 1, 1, 1), x, wt,
                         threads=4)
    d = lambda a: torch.from_numpy(a).cuda()
    res = None if res_scale is None else rng_s8(seed + 4, acc.shape)
    for name, epi, zp, lo, hi in _epilogues():
        if res is None:
            y = b2q.conv2d_s8(d(x), d(wt), d(bias), d(scale), p, epi)
            want = oracle.requant_s8(acc, bias, scale, zp, lo, hi)
        else:
            y = b2q.conv2d_s8_add(d(x), d(wt), d(bias), d(scale), d(res), res_scale, p, epi)
            want = oracle.requant_res_s8(acc, bias, scale, res, res_scale, zp, lo, hi)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), want, err_msg=name)
    return b2q.last_path()


@pytest.mark.parametrize("c,k", [(64, 256), (64, 64), (128, 96), (32, 48), (16, 256), (64, 192), (128, 144),
                                 (256, 400)])
def test_pointwise_short_reduction(cuda_lib, c, k):
    # narrow layers (G * K <= 256, G * C <= 256) run pixel-grouped, the others on plain tiles
    grouped = any(g * k <= 256 and g * c <= 256 for g in (2, 4, 8, 16))
    assert _case(4, 28, 28, c, 1, k, 0, 1, 2**15, seed=c + k) == ("tcgen05-tiled-grouped" if grouped else "tcgen05-tiled")


def test_im2col_short_reduction(cuda_lib):
    # 3x3 over 16 channels: reduction 144, im2col or packed GEMM
    _case(2, 40, 40, 16, 3, 64, 1, 1, 2**15, seed=5)


def test_large_bias(cuda_lib):
    # biases near 2^22 and 2^30 (the int32 sum wraps for the latter)
    _case(2, 28, 28, 64, 1, 128, 0, 1, 3 * 2**20, special=None, seed=11)
    _case(2, 28, 28, 64, 1, 128, 0, 1, 2**30, seed=12)


def test_nonfinite_scales(cuda_lib):
    special = {0: np.float32(np.nan), 1: np.float32(np.inf), 2: np.float32(-np.inf), 3: np.float32(2.0**101)}
    _case(2, 28, 28, 64, 1, 128, 0, 1, 2**15, special=special, seed=13)


@pytest.mark.parametrize("res_scale", [0.5, 0.0078125, 1e31])
def test_residual_add_short_reduction(cuda_lib, res_scale):
    _case(2, 28, 28, 64, 1, 256, 0, 1, 2**15, res_scale=res_scale, seed=17)


def test_bmm_short_reduction(cuda_lib):
    b2q = _b2q()
    batch, m, n, kk = 3, 300, 192, 64
    a = rng_s8(21, (batch, m, kk), -128, 127)
    b = rng_s8(22, (batch, kk, n), -128, 127)
    bias = np.random.default_rng(23).integers(-2**15, 2**15, size=n).astype(np.int32)
    scale = _scales(n, 24)
    acc = np.einsum("bmk,bkn->bmn", a.astype(np.int64), b.astype(np.int64)).astype(np.int32)
    d = lambda t: torch.from_numpy(t).cuda()
    for name, epi, zp, lo, hi in _epilogues():
        y = b2q.bmm_s8(d(a), d(b), 0, 0, epi, bias=d(bias), col_scale=d(scale))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), oracle.requant_s8(acc, bias, scale, zp, lo, hi),
                                      err_msg=name)


@pytest.mark.parametrize("n,hw,c,k,expect", [
    (4, 28, 32, 16, "tcgen05-tiled-grouped"),   # G = 8: rows of 256 channels, 128 outputs
    (3, 30, 16, 96, "tcgen05-tiled-grouped"),   # G = 2 (MobileNetV2 g2b1.expand shape)
    (2, 28, 64, 64, "tcgen05-tiled-grouped"),   # G = 4
    (1, 7, 32, 16, "tcgen05-tiled"),            # M = 49: no G divides it
])
def test_pixel_grouped_pointwise(cuda_lib, n, hw, c, k, expect):
    """1x1 convs of narrow layers as GEMMs over G-pixel rows with block-diagonal weights: every
    epilogue form, int32 / fp32 outputs and the fused residual add against the oracle."""
    b2q = _b2q()
    assert _case(n, hw, hw, c, 1, k, 0, 1, 2**15, seed=c * k + n) == expect
    _case(n, hw, hw, c, 1, k, 0, 1, 2**15, res_scale=0.5, seed=c * k + n + 1)
    x = rng_s8(9, (n, hw, hw, c), -128, 127)
    wt = rng_s8(10, (k, 1, 1, c), -128, 127)
    bias = np.random.default_rng(11).integers(-2**20, 2**20, size=k).astype(np.int32)
    scale = _scales(k, 12)
    acc = oracle.conv_s8(oracle.conv_args(n, hw, hw, c, 1, 1, k, 0, 0), x, wt, threads=4)
    d = lambda t: torch.from_numpy(t).cuda()
    p = b2q.Conv2DParams(0, 0, 1, 1, 1, 1, 1)
    y32 = b2q.conv2d_s8(d(x), d(wt), d(bias), None, p, b2q.Epilogue.int32())
    yf = b2q.conv2d_s8(d(x), d(wt), d(bias), d(scale), p, b2q.Epilogue.fp32())
    torch.cuda.synchronize()
    assert b2q.last_path() == expect
    np.testing.assert_array_equal(y32.cpu().numpy(), oracle.bias_add_i32(acc, bias))
    np.testing.assert_allclose(yf.cpu().numpy(), oracle.dequant_f32(acc, bias, scale), rtol=1e-5, atol=0)
