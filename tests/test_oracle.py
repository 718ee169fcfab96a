"""CPU tests: the oracle pinned to the reference's golden vectors, the requant / bmm / generator
semantics, and the host-side mirror of the reference interface.  No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.kat import kat_cases


def test_restated_oracle_matches_reference_goldens(golden):
    for kc in kat_cases(golden):
        a = oracle.conv_args(kc.n, kc.h, kc.w, kc.c, kc.r, kc.s, kc.k, kc.pad_h, kc.pad_w, kc.stride_h, kc.stride_w,
                             kc.dil_h, kc.dil_w, kc.groups, kc.by, kc.bx)
        y = oracle.conv_qi32(a, kc.x, kc.wt, kc.zp_in, kc.zp_f)
        np.testing.assert_array_equal(y, kc.y, err_msg=kc.name)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference oracle not built here")
def test_reference_oracle_reproduces_goldens(golden):
    for kc in kat_cases(golden):
        a = oracle.conv_args(kc.n, kc.h, kc.w, kc.c, kc.r, kc.s, kc.k, kc.pad_h, kc.pad_w, kc.stride_h, kc.stride_w,
                             kc.dil_h, kc.dil_w, kc.groups, kc.by, kc.bx)
        y = oracle.ref_conv_qi32(a, kc.kind, kc.x, kc.wt, kc.zp_in, kc.zp_f, kc.blocked)
        np.testing.assert_array_equal(y, kc.y, err_msg=kc.name)


def test_int8_oracle_equals_float_code_oracle():
    rng = np.random.default_rng(1)
    for (n, h, w, c, r, s, k, ph, pw, sh, sw, dh, dw, g) in [
        (2, 9, 8, 8, 3, 3, 6, 1, 1, 1, 1, 1, 1, 1),
        (1, 11, 10, 12, 3, 3, 8, 2, 1, 2, 2, 1, 2, 4),
        (2, 6, 6, 5, 1, 1, 3, 0, 0, 1, 1, 1, 1, 1),
    ]:
        x = rng.integers(-127, 128, size=(n, h, w, c)).astype(np.int8)
        wt = rng.integers(-127, 128, size=(k, r, s, c // g)).astype(np.int8)
        a = oracle.conv_args(n, h, w, c, r, s, k, ph, pw, sh, sw, dh, dw, g)
        y8 = oracle.conv_s8(a, x, wt, threads=2)
        yf = oracle.conv_qi32(a, x.astype(np.float32), wt.astype(np.float32), np.zeros(n, np.int32), 0)
        np.testing.assert_array_equal(y8, yf)


def test_int8_oracle_against_numpy_direct():
    rng = np.random.default_rng(2)
    n, h, w, c, k = 2, 6, 7, 8, 5
    x = rng.integers(-127, 128, size=(n, h, w, c)).astype(np.int8)
    wt = rng.integers(-127, 128, size=(k, 3, 3, c)).astype(np.int8)
    xp = np.pad(x.astype(np.int64), ((0, 0), (1, 1), (1, 1), (0, 0)))
    ref = np.zeros((n, h, w, k), np.int64)
    for r in range(3):
        for s in range(3):
            ref += np.einsum("nhwc,kc->nhwk", xp[:, r:r + h, s:s + w, :], wt[:, r, s, :].astype(np.int64))
    np.testing.assert_array_equal(oracle.conv_s8(oracle.conv_args(n, h, w, c, 3, 3, k), x, wt), ref)


def test_requant_round_half_even_and_clamp():
    acc = np.array([[5, 15, 25, -5, -15, 1000, -1000, 7]], dtype=np.int32)
    scale = np.array([0.1] * 8, dtype=np.float32)
    # float32(0.1) * 5 rounds to exactly 0.5 in fp32 -> half-even gives 0
    q = oracle.requant_s8(acc, None, scale)
    p = (acc.astype(np.float32) * scale).astype(np.float32)
    expect = np.clip(np.rint(p), -128, 127).astype(np.int8)
    np.testing.assert_array_equal(q, expect)
    # ReLU / ReLU6 as clamps, output zero point
    q2 = oracle.requant_s8(acc, np.full(8, 3, np.int32), np.full(8, 0.5, np.float32), zp=2, lo=2, hi=20)
    t = (acc.astype(np.int64) + 3).astype(np.float32) * np.float32(0.5)
    expect2 = (np.rint(np.clip(t, 0, 18)) + 2).astype(np.int8)
    np.testing.assert_array_equal(q2, expect2)


def test_requant_nonfinite_rules():
    # rint_sat: NaN -> 0 before the clamp; +-inf and huge values saturate to the bounds
    acc = np.array([[0, 5, -5, 2**30]], dtype=np.int32)
    scale = np.array([np.inf, np.inf, np.inf, 1e30], dtype=np.float32)
    q = oracle.requant_s8(acc, None, scale)
    np.testing.assert_array_equal(q, np.array([[0, 127, -128, 127]], dtype=np.int8))
    q2 = oracle.requant_s8(acc, None, scale, zp=0, lo=3, hi=9)
    np.testing.assert_array_equal(q2, np.array([[3, 9, 3, 9]], dtype=np.int8))


def test_requant_bias_wraps_int32():
    acc = np.array([[2**31 - 1]], dtype=np.int32)
    q = oracle.dequant_f32(acc, np.array([1], np.int32), np.array([1.0], np.float32))
    assert q[0, 0] == np.float32(-2.0**31)


def test_bmm_i32_oracle_wraps_like_int32():
    rng = np.random.default_rng(3)
    for ta in (0, 1):
        for tb in (0, 1):
            batch, M, N, K = 2, 5, 7, 9
            A = rng.integers(-2**31, 2**31, size=(batch, K, M) if ta else (batch, M, K), dtype=np.int64)
            B = rng.integers(-2**31, 2**31, size=(batch, N, K) if tb else (batch, K, N), dtype=np.int64)
            C = oracle.bmm_i32(A.astype(np.int32), B.astype(np.int32), batch, M, N, K, ta, tb)
            Am = np.swapaxes(A, 1, 2) if ta else A
            Bm = np.swapaxes(B, 1, 2) if tb else B
            ref = np.zeros((batch, M, N), dtype=np.uint64)
            for kk in range(K):  # exact mod 2^64, then truncate to 32 bits
                ref += (Am[:, :, kk:kk + 1].astype(np.uint64) * Bm[:, kk:kk + 1, :].astype(np.uint64))
            np.testing.assert_array_equal(C, (ref & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.int32))


def test_bmm_s8_oracle_matches_numpy():
    rng = np.random.default_rng(4)
    for ta in (0, 1):
        for tb in (0, 1):
            batch, M, N, K = 3, 17, 19, 13
            A = rng.integers(-127, 128, size=(batch, K, M) if ta else (batch, M, K)).astype(np.int8)
            B = rng.integers(-127, 128, size=(batch, N, K) if tb else (batch, K, N)).astype(np.int8)
            C = oracle.bmm_s8(A, B, batch, M, N, K, ta, tb, threads=2)
            Am = np.swapaxes(A, 1, 2) if ta else A
            Bm = np.swapaxes(B, 1, 2) if tb else B
            np.testing.assert_array_equal(C, np.matmul(Am.astype(np.int64), Bm.astype(np.int64)))


def test_generators_agree_between_c_and_python():
    from my_own_cnn_b200 import synth

    for seed, tid, lo, hi in [(42, 1, -127, 127), (7, 99, 0, 127), (1, 2, -3, 3)]:
        a = oracle.fill_s8_uniform(seed, tid, lo, hi, 1000, 5000)
        b = synth.s8_uniform_host(seed, tid, lo, hi, 1000, 5000)
        np.testing.assert_array_equal(a, b)
        assert a.min() >= lo and a.max() <= hi
    a = oracle.fill_i32_uniform(5, 3, -2**15, 2**15, 0, 4096)
    np.testing.assert_array_equal(a, synth.i32_uniform_host(5, 3, -2**15, 2**15, 0, 4096))
    tab = synth.quantile_table("normal", 30.0, -127, 127)
    np.testing.assert_array_equal(oracle.fill_s8_table(9, 4, tab, 77, 3000), synth.s8_table_host(9, 4, tab, 77, 3000))
    np.testing.assert_array_equal(oracle.fill_f32_uniform(3, 8, 1e-4, 1e-3, 0, 300), synth.scales_f32(300, 3, 8))


def test_quantile_tables():
    from my_own_cnn_b200 import synth

    t = synth.quantile_table("normal", 30.0, -127, 127).astype(np.float64)
    assert abs(t.mean()) < 0.01 and 29.0 < t.std() < 31.0
    hn = synth.quantile_table("halfnormal", 40.0, 0, 127).astype(np.float64)
    assert hn.min() >= 0 and hn.max() == 127
    assert 40.0 * 0.75 < hn.mean() < 40.0 * 0.85  # E|N(0,s)| = s*sqrt(2/pi) ~ 0.798 s (before clipping)


def test_uniform_distribution_moments():
    v = oracle.fill_s8_uniform(42, 1, -127, 127, 0, 200000).astype(np.float64)
    assert abs(v.mean()) < 0.5
    assert abs(v.std() - np.sqrt((255**2 - 1) / 12)) < 0.5


def test_residual_requant_oracle():
    """Residual add: p = fl(fl(t) * s) + fl(res * rs) in fp32, then the int8 requant rules.
    res = 0 reduces to the plain requant; a numpy restatement with float32 steps agrees."""
    rng = np.random.default_rng(11)
    acc = rng.integers(-2**20, 2**20, size=(37, 24), dtype=np.int64).astype(np.int32)
    bias = rng.integers(-2**15, 2**15, size=24, dtype=np.int64).astype(np.int32)
    scale = rng.uniform(1e-4, 1e-3, size=24).astype(np.float32)
    zero = np.zeros(acc.shape, dtype=np.int8)
    np.testing.assert_array_equal(oracle.requant_res_s8(acc, bias, scale, zero, 0.7),
                                  oracle.requant_s8(acc, bias, scale))
    res = rng.integers(-128, 128, size=acc.shape, dtype=np.int64).astype(np.int8)
    rs = np.float32(0.37)
    for lo, hi in [(-128, 127), (0, 127), (0, 96)]:
        got = oracle.requant_res_s8(acc, bias, scale, res, float(rs), 0, lo, hi)
        t = (acc.astype(np.int64) + bias).astype(np.int32)
        p = (t.astype(np.float32) * scale).astype(np.float32) + (res.astype(np.float32) * rs).astype(np.float32)
        want = np.clip(np.rint(p.astype(np.float32)), lo, hi).astype(np.int8)
        np.testing.assert_array_equal(got, want)


def test_pool_oracles_against_numpy():
    rng = np.random.default_rng(12)
    x = rng.integers(-128, 128, size=(2, 9, 11, 24), dtype=np.int64).astype(np.int8)
    y = oracle.maxpool_s8(x, 3, 3, 2, 2, 1, 1)
    assert y.shape == (2, 5, 6, 24)
    xp = np.pad(x.astype(np.int32), ((0, 0), (1, 1), (1, 1), (0, 0)), constant_values=-1000)
    want = np.full(y.shape, -1000, dtype=np.int32)
    for i in range(3):
        for j in range(3):
            want = np.maximum(want, xp[:, i:i + 9:2, j:j + 11:2, :][:, :5, :6, :])
    np.testing.assert_array_equal(y, want.astype(np.int8))
    a = oracle.global_avgpool_s8(x)
    s = x.astype(np.int32).sum(axis=(1, 2))
    want = np.clip(np.rint(s.astype(np.float32) / np.float32(99)), -128, 127).astype(np.int8)
    np.testing.assert_array_equal(a, want)


@pytest.mark.parametrize("case", [
    # n, h, w, c, k, r, s, pad_h, pad_w, sh, sw, dh, dw, groups, by, bx
    (2, 7, 6, 4, 6, 3, 2, 1, 0, 1, 1, 1, 1, 2, 1, 1),
    (1, 9, 9, 6, 4, 3, 3, 2, 2, 2, 2, 2, 2, 1, 1, 1),
    (2, 6, 6, 4, 5, 3, 3, 1, 1, 1, 1, 1, 1, 1, 2, 3),
    (2, 8, 8, 6, 6, 3, 3, 1, 1, 1, 1, 1, 1, 3, 2, 2),
])
@pytest.mark.parametrize("mode", [0, 1])
def test_f32_restatement_matches_reference_cpu(case, mode):
    """oracle/f32_oracle.py (float64) against the reference's own fp32 loops (src/cpu_ref.cpp:116-371):
    equal within fp32 rounding of the reference's sums, dbias included."""
    from oracle import f32_oracle

    if not oracle.ref_available():
        pytest.skip("reference oracle not built")
    n, h, w, c, k, r, s, ph, pw, sh, sw, dh, dw, G, by, bx = case
    prm = (ph, pw, sh, sw, dh, dw, G)
    blocked = by * bx > 1
    rng = np.random.default_rng(sum(case) + mode)
    ho, wo = f32_oracle.out_hw(h, w, r, s, ph, pw, sh, sw, dh, dw)
    x = rng.standard_normal((n, h, w, c)).astype(np.float32)
    wt = rng.standard_normal((k, by, bx, r, s, c // G) if blocked else (k, r, s, c // G)).astype(np.float32)
    dy = rng.standard_normal((n, ho, wo, k)).astype(np.float32)
    bias = rng.standard_normal(k * by * bx).astype(np.float32) if blocked else None
    a = oracle.conv_args(n, h, w, c, r, s, k, *prm, by, bx)
    ye, yb = f32_oracle.fprop(x, wt, prm, by, bx, bias, mode)
    y = oracle.ref_conv_f32(a, 0, blocked, x, wt, (n, ho, wo, k), None if bias is None else bias.copy(), mode)
    assert (np.abs(y - ye) <= 1e-5 * yb + 1e-6).all()
    dxe, dxb = f32_oracle.bprop(dy, wt, (n, h, w, c), prm, by, bx)
    dx = oracle.ref_conv_f32(a, 1, blocked, dy, wt, (n, h, w, c))
    assert (np.abs(dx - dxe) <= 1e-5 * dxb + 1e-6).all()
    dwe, dwb, dbe = f32_oracle.grad(x, dy, r, s, prm, by, bx, mode)
    db = np.zeros(k * by * bx, np.float32)
    dwr = oracle.ref_conv_f32(a, 2, blocked, x, dy, dwe.shape, db if blocked else None, mode)
    assert (np.abs(dwr - dwe) <= 1e-5 * dwb + 1e-6).all()
    if blocked:
        np.testing.assert_allclose(db, dbe, rtol=1e-5, atol=1e-4)
