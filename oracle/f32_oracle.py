"""float64 restatement of the reference's fp32 convolution loops -- TEST INFRASTRUCTURE ONLY.

Only tests/ may use this module, as the checker of the fp32 tensor-core paths.  It follows
src/cpu_ref.cpp of NikitaYak02/my_own_cnn:
  fprop         cpu_fprop_nhwc        (cpu_ref.cpp:116-148)
  bprop         cpu_bprop_nhwc        (cpu_ref.cpp:150-192)
  grad          cpu_grad_nhwc         (cpu_ref.cpp:194-230)
  blocked fprop cpu_block_fprop_nhwc  (cpu_ref.cpp:232-271, bias index conv_types.h:184-188)
  blocked bprop cpu_block_bprop_nhwc  (cpu_ref.cpp:273-316)
  blocked grad  cpu_block_grad_nhwc   (cpu_ref.cpp:318-371, including its dbias rule)
but sums in float64 and also returns, for every output element, the sum of the absolute values of
the products that make it up: the error bound of an fp32 result is a multiple of that sum.
Blocks: the output is cut into by x bx equal blocks (ho / by rows, wo / bx columns); block (i, j)
uses filter slice w[:, i, j].
"""
from __future__ import annotations

import numpy as np


def out_hw(h, w, r, s, pad_h, pad_w, sh, sw, dh, dw):
    return (h + 2 * pad_h - dh * (r - 1) - 1) // sh + 1, (w + 2 * pad_w - dw * (s - 1) - 1) // sw + 1


def _cols(x, r, s, pad_h, pad_w, sh, sw, dh, dw):
    """im2col: [n, ho, wo, r, s, c] float64, zero in the padding."""
    n, h, w, c = x.shape
    ho, wo = out_hw(h, w, r, s, pad_h, pad_w, sh, sw, dh, dw)
    xp = np.zeros((n, h + 2 * pad_h, w + 2 * pad_w, c), dtype=np.float64)
    xp[:, pad_h:pad_h + h, pad_w:pad_w + w] = x
    out = np.empty((n, ho, wo, r, s, c), dtype=np.float64)
    for i in range(r):
        for j in range(s):
            out[:, :, :, i, j] = xp[:, i * dh: i * dh + sh * (ho - 1) + 1: sh, j * dw: j * dw + sw * (wo - 1) + 1: sw]
    return out


def _blocks(ho, wo, by, bx):
    bh, bw = ho // by, wo // bx
    for i in range(by):
        for j in range(bx):
            yield i, j, slice(i * bh, (i + 1) * bh), slice(j * bw, (j + 1) * bw)


def fprop(x, w, prm, by=1, bx=1, bias=None, bias_mode=0):
    """x [n,h,w,c]; w [k,r,s,cg] or [k,by,bx,r,s,cg]; prm = (pad_h, pad_w, sh, sw, dh, dw, groups).
    Returns (y, bound) float64 [n,ho,wo,k]."""
    pad_h, pad_w, sh, sw, dh, dw, groups = prm
    wt = np.asarray(w, np.float64)
    if wt.ndim == 4:
        wt = wt[:, None, None]
    k, _, _, r, s, cg = wt.shape
    cols = _cols(np.asarray(x, np.float64), r, s, pad_h, pad_w, sh, sw, dh, dw)
    n, ho, wo = cols.shape[:3]
    kg = k // groups
    y = np.zeros((n, ho, wo, k))
    bound = np.zeros((n, ho, wo, k))
    for i, j, rs, cs in _blocks(ho, wo, by, bx):
        blk = cols[:, rs, cs]
        for g in range(groups):
            a = blk[..., g * cg:(g + 1) * cg].reshape(blk.shape[:3] + (-1,))
            b = wt[g * kg:(g + 1) * kg, i, j].reshape(kg, -1)
            y[:, rs, cs, g * kg:(g + 1) * kg] = a @ b.T
            bound[:, rs, cs, g * kg:(g + 1) * kg] = np.abs(a) @ np.abs(b).T
        if bias is not None:
            nb = by * bx
            idx = np.arange(k) * nb + (i * bx + j if bias_mode == 0 else 0)
            y[:, rs, cs] += np.asarray(bias, np.float64)[idx]
            bound[:, rs, cs] += np.abs(np.asarray(bias, np.float64)[idx])
    return y, bound


def bprop(dy, w, in_shape, prm, by=1, bx=1):
    """dx for dy [n,ho,wo,k]; in_shape = (n,h,w,c).  Returns (dx, bound) float64."""
    pad_h, pad_w, sh, sw, dh, dw, groups = prm
    wt = np.asarray(w, np.float64)
    if wt.ndim == 4:
        wt = wt[:, None, None]
    k, _, _, r, s, cg = wt.shape
    n, h, wd, c = in_shape
    dyf = np.asarray(dy, np.float64)
    ho, wo = dyf.shape[1:3]
    kg = k // groups
    # col[n, ho, wo, r, s, c] = sum_k dy * w (per block / group), then scatter-add over the taps
    col = np.zeros((n, ho, wo, r, s, c))
    colb = np.zeros((n, ho, wo, r, s, c))
    for i, j, rs, cs in _blocks(ho, wo, by, bx):
        for g in range(groups):
            a = dyf[:, rs, cs, g * kg:(g + 1) * kg]
            b = wt[g * kg:(g + 1) * kg, i, j]  # [kg, r, s, cg]
            col[:, rs, cs, :, :, g * cg:(g + 1) * cg] = np.tensordot(a, b, axes=([3], [0]))
            colb[:, rs, cs, :, :, g * cg:(g + 1) * cg] = np.tensordot(np.abs(a), np.abs(b), axes=([3], [0]))
    dxp = np.zeros((n, h + 2 * pad_h, wd + 2 * pad_w, c))
    bp = np.zeros_like(dxp)
    for ri in range(r):
        for sj in range(s):
            sl = (slice(None), slice(ri * dh, ri * dh + sh * (ho - 1) + 1, sh),
                  slice(sj * dw, sj * dw + sw * (wo - 1) + 1, sw))
            dxp[sl] += col[:, :, :, ri, sj]
            bp[sl] += colb[:, :, :, ri, sj]
    return dxp[:, pad_h:pad_h + h, pad_w:pad_w + wd], bp[:, pad_h:pad_h + h, pad_w:pad_w + wd]


def grad(x, dy, r, s, prm, by=1, bx=1, bias_mode=0):
    """dw [k,by,bx,r,s,cg] (squeezed to [k,r,s,cg] when by = bx = 1), its bound, and dbias
    [k*by*bx] by the reference's rule (tap (0, 0) inside the image)."""
    pad_h, pad_w, sh, sw, dh, dw_, groups = prm
    xf = np.asarray(x, np.float64)
    dyf = np.asarray(dy, np.float64)
    n, h, wd, c = xf.shape
    k = dyf.shape[3]
    cg, kg = c // groups, k // groups
    cols = _cols(xf, r, s, pad_h, pad_w, sh, sw, dh, dw_)
    ho, wo = cols.shape[1:3]
    dwt = np.zeros((k, by, bx, r, s, cg))
    bound = np.zeros_like(dwt)
    dbias = np.zeros(k * by * bx)
    for i, j, rs, cs in _blocks(ho, wo, by, bx):
        for g in range(groups):
            a = dyf[:, rs, cs, g * kg:(g + 1) * kg].reshape(-1, kg)
            b = cols[:, rs, cs, :, :, g * cg:(g + 1) * cg].reshape(a.shape[0], -1)
            dwt[g * kg:(g + 1) * kg, i, j] = (a.T @ b).reshape(kg, r, s, cg)
            bound[g * kg:(g + 1) * kg, i, j] = (np.abs(a).T @ np.abs(b)).reshape(kg, r, s, cg)
        # dbias: output pixels whose tap (0, 0) input is inside the image
        hos = np.arange(ho)[rs]
        wos = np.arange(wo)[cs]
        vh = (hos * sh - pad_h >= 0) & (hos * sh - pad_h < h)
        vw = (wos * sw - pad_w >= 0) & (wos * sw - pad_w < wd)
        part = dyf[:, rs, cs][:, vh][:, :, vw].sum(axis=(0, 1, 2))
        idx = np.arange(k) * by * bx + (i * bx + j if bias_mode == 0 else 0)
        dbias[idx] += part
    if by == 1 and bx == 1:
        return dwt[:, 0, 0], bound[:, 0, 0], dbias
    return dwt, bound, dbias


def bmm(A, B, ta, tb):
    """C = op(A) @ op(B) per batch item in float64, and the bound sum |a||b|."""
    a = np.asarray(A, np.float64)
    b = np.asarray(B, np.float64)
    if ta:
        a = a.transpose(0, 2, 1)
    if tb:
        b = b.transpose(0, 2, 1)
    return a @ b, np.abs(a) @ np.abs(b)
