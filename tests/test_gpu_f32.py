"""fp32 drop-ins on the tensor cores (3 x TF32 split products): conv fprop / bprop / grad, regular
and blocked (with both bias modes), and the fp32 bmm with its layer API.

Tolerance (fp32 results, written here): |got - exact| <= 1e-5 * sum(|a| * |b|) over the products
that make up each element (plus 1e-30), where `exact` is the float64 restatement of the reference's
loops (oracle/f32_oracle.py).  The reference's own fp32 CPU loops (src/cpu_ref.cpp, compiled from
its sources) are held to the same bound, and the reference's unmodified conv_bench driver, linked
against this library, must pass its own --check."""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import f32_oracle, oracle

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
REL = 1e-5


def _b2q():
    import my_own_cnn_b200 as b2q

    return b2q


def _close(got, exact, bound, what):
    err = np.abs(np.asarray(got, np.float64) - exact)
    lim = REL * bound + 1e-30
    bad = err > lim
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside 1e-5 * sum|ab|; worst {err[bad].max():.3e}"


def _rand(seed, shape, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


CASES = [
    # n, h, w, c, k, r, s, pad_h, pad_w, sh, sw, dh, dw, groups
    (2, 20, 20, 32, 48, 3, 3, 1, 1, 1, 1, 1, 1, 1),
    (1, 56, 56, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1),      # BASELINE config 1 geometry
    (2, 17, 23, 12, 20, 5, 3, 2, 1, 2, 1, 1, 1, 1),      # odd sizes, stride 2 on H, C % 4 != 0
    (2, 16, 16, 32, 32, 3, 3, 2, 2, 1, 1, 2, 2, 1),      # dilation 2
    (2, 14, 14, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 4),      # groups 4
    (2, 12, 12, 32, 32, 3, 3, 1, 1, 2, 2, 1, 1, 32),     # depthwise, stride 2
    (3, 9, 9, 256, 96, 1, 1, 0, 0, 1, 1, 1, 1, 1),       # pointwise, K = 96
    (1, 23, 23, 3, 64, 7, 7, 3, 3, 2, 2, 1, 1, 1),       # stem
    # inputs >= 128 KiB with C % 4 == 0: im2col TMA over hi / lo copies (fprop; bprop when stride 1)
    (4, 28, 28, 64, 96, 3, 3, 1, 1, 2, 2, 1, 1, 1),      # stride 2
    (2, 32, 32, 48, 64, 5, 5, 2, 2, 1, 1, 1, 1, 1),      # 5x5
    (2, 40, 40, 32, 32, 3, 3, 2, 2, 1, 1, 2, 2, 1),      # dilation 2
    (2, 40, 40, 36, 40, 3, 3, 1, 0, 1, 1, 1, 1, 1),      # C = 36 (channel padding to 64), asymmetric pad
    (2, 28, 28, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 4),      # groups 4 on the im2col route (group = batch item)
    (2, 24, 24, 72, 48, 3, 3, 1, 1, 1, 1, 1, 1, 2),      # groups 2, 36 channels per group
]


@pytest.mark.parametrize("policy", [0, 1])
@pytest.mark.parametrize("case", CASES)
def test_fprop_bprop_grad(cuda_lib, case, policy):
    """policy 0: automatic (tensor cores; CUDA cores for groups of at most 16 channel pairs);
    policy 1: the CUDA-core kernels for every case (cross-check of the two datapaths)."""
    b2q = _b2q()
    b2q.set_path_policy(policy)
    try:
        _fprop_bprop_grad(b2q, case, policy)
    finally:
        b2q.set_path_policy(0)


def _fprop_bprop_grad(b2q, case, policy):
    n, h, w, c, k, r, s, ph, pw, sh, sw, dh, dw, G = case
    prm = (ph, pw, sh, sw, dh, dw, G)
    p = b2q.Conv2DParams(*prm)
    ho, wo = b2q.conv_out_shape(h, w, c, r, s, k, p)
    x = _rand(sum(case), (n, h, w, c))
    wt = _rand(sum(case) + 1, (k, r, s, c // G))
    dy = _rand(sum(case) + 2, (n, ho, wo, k))
    cu = lambda a: torch.from_numpy(a).cuda()
    y = torch.full((n, ho, wo, k), float("nan"), device="cuda")
    dx = torch.full((n, h, w, c), float("nan"), device="cuda")
    dwt = torch.full((k, r, s, c // G), float("nan"), device="cuda")
    b2q.launch_fprop_nhwc(cu(x), cu(wt), y, n, h, w, c, r, s, k, p)
    direct = policy == 1 or (c // G) * (k // G) <= 16
    assert b2q.last_path() == ("cuda-core-f32" if direct else "tcgen05-f32")
    b2q.launch_bprop_nhwc(cu(dy), cu(wt), dx, n, h, w, c, r, s, k, p)
    b2q.launch_grad_nhwc(cu(x), cu(dy), dwt, n, h, w, c, r, s, k, p)
    torch.cuda.synchronize()
    ye, yb = f32_oracle.fprop(x, wt, prm)
    _close(y.cpu().numpy(), ye, yb, f"fprop {case}")
    dxe, dxb = f32_oracle.bprop(dy, wt, (n, h, w, c), prm)
    _close(dx.cpu().numpy(), dxe, dxb, f"bprop {case}")
    dwe, dwb, _ = f32_oracle.grad(x, dy, r, s, prm)
    _close(dwt.cpu().numpy(), dwe, dwb, f"grad {case}")
    if policy == 0 and oracle.ref_available() and n * ho * wo * k * r * s * c // G < 5e7:
        a = oracle.conv_args(n, h, w, c, r, s, k, *prm)
        _close(oracle.ref_conv_f32(a, 0, False, x, wt, (n, ho, wo, k)), ye, yb, "reference fprop")
        _close(oracle.ref_conv_f32(a, 1, False, dy, wt, (n, h, w, c)), dxe, dxb, "reference bprop")
        _close(oracle.ref_conv_f32(a, 2, False, x, dy, (k, r, s, c // G)), dwe, dwb, "reference grad")


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("case", [
    # n, h, w, c, k, r, pad, stride, groups, by, bx
    (2, 12, 12, 16, 24, 3, 1, 1, 1, 2, 3),
    (3, 16, 12, 32, 32, 3, 1, 2, 2, 2, 2),
    (2, 8, 8, 24, 16, 1, 0, 1, 1, 4, 4),
    (2, 8, 8, 8, 8, 3, 1, 1, 8, 2, 2),      # depthwise: the CUDA-core fp32 kernels
])
def test_blocked_with_bias(cuda_lib, case, mode):
    b2q = _b2q()
    n, h, w, c, k, r, pad, st, G, by, bx = case
    prm = (pad, pad, st, st, 1, 1, G)
    bp = b2q.BlockConv2DParams(b2q.Conv2DParams(*prm), by, bx)
    ho, wo = b2q.conv_out_shape(h, w, c, r, r, k, bp.conv)
    x = _rand(sum(case) + mode, (n, h, w, c))
    wt = _rand(sum(case) + 7, (k, by, bx, r, r, c // G))
    bias = _rand(sum(case) + 8, (k * by * bx,))
    dy = _rand(sum(case) + 9, (n, ho, wo, k))
    cu = lambda a: torch.from_numpy(a).cuda()
    y = torch.full((n, ho, wo, k), float("nan"), device="cuda")
    dx = torch.full((n, h, w, c), float("nan"), device="cuda")
    dwt = torch.full((k, by, bx, r, r, c // G), float("nan"), device="cuda")
    dbias = torch.full((k * by * bx,), float("nan"), device="cuda")
    bm = b2q.BlockBiasMode(mode)
    b2q.launch_block_fprop_nhwc(cu(x), cu(wt), y, n, h, w, c, r, r, k, bp, cu(bias), bm)
    b2q.launch_block_bprop_nhwc(cu(dy), cu(wt), dx, n, h, w, c, r, r, k, bp)
    b2q.launch_block_grad_nhwc(cu(x), cu(dy), dwt, n, h, w, c, r, r, k, bp, dbias, bm)
    torch.cuda.synchronize()
    ye, yb = f32_oracle.fprop(x, wt, prm, by, bx, bias, mode)
    _close(y.cpu().numpy(), ye, yb, "blocked fprop")
    dxe, dxb = f32_oracle.bprop(dy, wt, (n, h, w, c), prm, by, bx)
    _close(dx.cpu().numpy(), dxe, dxb, "blocked bprop")
    dwe, dwb, dbe = f32_oracle.grad(x, dy, r, r, prm, by, bx, mode)
    _close(dwt.cpu().numpy(), dwe, dwb, "blocked grad")
    _close(dbias.cpu().numpy(), dbe, np.abs(dbe) + 1e-3 * np.abs(dy).sum(), "blocked dbias")
    if oracle.ref_available():
        a = oracle.conv_args(n, h, w, c, r, r, k, *prm, by, bx)
        _close(oracle.ref_conv_f32(a, 0, True, x, wt, (n, ho, wo, k), bias.copy(), mode), ye, yb, "reference fprop")
        db_ref = np.zeros(k * by * bx, np.float32)
        dw_ref = oracle.ref_conv_f32(a, 2, True, x, dy, (k, by, bx, r, r, c // G), db_ref, mode)
        _close(dw_ref, dwe, dwb, "reference grad")
        np.testing.assert_allclose(db_ref, dbe, rtol=1e-4, atol=1e-3)


def test_grad_long_reduction_split(cuda_lib):
    """A filter gradient reduced over 100352 output pixels (split across SMs, then summed)."""
    b2q = _b2q()
    n, h, w, c, k = 32, 56, 56, 64, 64
    prm = (1, 1, 1, 1, 1, 1, 1)
    p = b2q.Conv2DParams(*prm)
    x = _rand(1, (n, h, w, c))
    dy = _rand(2, (n, h, w, k))
    dwt = torch.empty((k, 3, 3, c), device="cuda")
    b2q.launch_grad_nhwc(torch.from_numpy(x).cuda(), torch.from_numpy(dy).cuda(), dwt, n, h, w, c, 3, 3, k, p)
    torch.cuda.synchronize()
    dwe, dwb, _ = f32_oracle.grad(x, dy, 3, 3, prm)
    _close(dwt.cpu().numpy(), dwe, dwb, "long grad")


@pytest.mark.parametrize("dims", [(1, 1, 1, 1), (2, 17, 19, 13), (3, 128, 96, 64), (2, 300, 260, 700), (1, 8, 8, 0)])
def test_bmm_f32_transposes(cuda_lib, dims):
    b2q = _b2q()
    batch, M, N, K = dims
    for ta in (0, 1):
        for tb in (0, 1):
            A = _rand(M + ta, (batch, K, M) if ta else (batch, M, K))
            B = _rand(N + tb, (batch, N, K) if tb else (batch, K, N))
            C = torch.full((batch, M, N), float("nan"), device="cuda")
            b2q.bmm_matmul(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), C, batch, M, N, K, ta, tb)
            torch.cuda.synchronize()
            ce, cb = f32_oracle.bmm(A, B, ta, tb)
            _close(C.cpu().numpy(), ce, cb, f"bmm {dims} ta={ta} tb={tb}")


def test_bmm_layer_api(cuda_lib):
    """bmm_fprop / bmm_bprop (bmm.h:41-66): Y = A B^T, dA = dY B, dB = dY^T A."""
    b2q = _b2q()
    N, W, H, C = 3, 40, 24, 56
    A, B, dY = _rand(1, (N, W, C)), _rand(2, (N, H, C)), _rand(3, (N, W, H))
    cu = lambda a: torch.from_numpy(a).cuda()
    Y, dA, dB = (torch.empty(sh, device="cuda") for sh in ((N, W, H), (N, W, C), (N, H, C)))
    b2q.bmm_fprop(cu(A), cu(B), Y, N, W, H, C)
    b2q.bmm_bprop(cu(A), cu(B), cu(dY), dA, dB, N, W, H, C)
    torch.cuda.synchronize()
    _close(Y.cpu().numpy(), *f32_oracle.bmm(A, B, 0, 1), "bmm_fprop")
    _close(dA.cpu().numpy(), *f32_oracle.bmm(dY, B, 0, 0), "bmm_bprop_dA")
    _close(dB.cpu().numpy(), *f32_oracle.bmm(dY, A, 1, 0), "bmm_bprop_dB")


@pytest.mark.parametrize("args", [
    ["--op", "all", "--n", "2", "--h", "20", "--w", "20", "--c", "32", "--k", "48"],
    ["--op", "all", "--n", "2", "--h", "14", "--w", "14", "--c", "64", "--k", "64", "--groups", "4", "--stride_h", "2",
     "--stride_w", "2"],
    ["--op", "all", "--custom_mode", "blocked", "--n", "2", "--h", "12", "--w", "12", "--c", "16", "--k", "24",
     "--block_by", "2", "--block_bx", "3"],
])
def test_reference_conv_bench_links_and_checks(cuda_lib, args):
    """The reference's unmodified fp32 conv_bench (src/main.cpp), linked against the shim, passes its
    own --check of fprop / bprop / grad against its CPU loops."""
    binary = ROOT / "oracle" / "_ref" / "conv_bench_b200"
    if not binary.exists():
        pytest.skip("conv_bench not built (needs the reference sources at build time)")
    proc = subprocess.run([str(binary), *args, "--check", "--warmup", "1", "--iters", "3"], capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    checks = [ln for ln in proc.stdout.splitlines() if ln.startswith("check ")]
    assert len(checks) == 3, proc.stdout
    assert all("pass=yes" in ln for ln in checks), proc.stdout
