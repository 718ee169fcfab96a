"""CPU check of the algebra behind the quantized-int32 drop-in's tensor-core route (no GPU).

The route multiplies raw 8-bit codes (padding taps carry the image's own input zero point) and
restores the zero points with one term per packed row and one per filter row:
    sum (a - zx)(b - zw) = sum ab - zw * sum a - zx * sum b + T * zx * zw     (mod 2^32)
This file restates that decomposition in numpy -- im2col with zx in the padding, per-row term
T*zx*zw - zw*sum(a), per-column sum(b), one int64 GEMM per (block, group) -- and checks it against
the C oracle's direct loop (oracle.c, itself pinned to the reference's cpu_ref.cpp) on blocked,
grouped, strided and padded geometries with both U8 and S5 code ranges."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle


def _decomposed(x, w, zin, zf, n, h, wd, c, r, s, k, prm, by=1, bx=1):
    pad_h, pad_w, sh, sw, dh, dw, G = prm
    ho = (h + 2 * pad_h - dh * (r - 1) - 1) // sh + 1
    wo = (wd + 2 * pad_w - dw * (s - 1) - 1) // sw + 1
    cg, kg = c // G, k // G
    T = r * s * cg
    wt = w.reshape(k, by, bx, r, s, cg).astype(np.int64)
    y = np.zeros((n, ho, wo, k), dtype=np.int64)
    bh, bw = ho // by, wo // bx
    for img in range(n):
        # padded input with the image's zero point in the padding
        xp = np.full((h + 2 * pad_h, wd + 2 * pad_w, c), zin[img], dtype=np.int64)
        xp[pad_h:pad_h + h, pad_w:pad_w + wd] = x[img]
        for oy in range(ho):
            for ox in range(wo):
                blk_y, blk_x = oy // bh, ox // bw
                taps = np.stack([xp[oy * sh + i * dh, ox * sw + j * dw] for i in range(r) for j in range(s)])
                for g in range(G):
                    a = taps[:, g * cg:(g + 1) * cg].reshape(-1)  # [T]
                    b = wt[g * kg:(g + 1) * kg, blk_y, blk_x].reshape(kg, -1)  # [kg, T]
                    rowterm = T * zin[img] * zf - zf * a.sum()
                    colsum = b.sum(axis=1)
                    y[img, oy, ox, g * kg:(g + 1) * kg] = b @ a + rowterm - zin[img] * colsum
    return ((y + 2**31) % 2**32 - 2**31).astype(np.int32)


@pytest.mark.parametrize("case", [
    # kind, n, h, w, c, r, s, k, prm (pad_h, pad_w, sh, sw, dh, dw, groups), by, bx
    (0, 2, 6, 7, 4, 3, 3, 6, (1, 1, 1, 1, 1, 1, 1), 1, 1),
    (1, 2, 6, 6, 4, 3, 3, 5, (1, 1, 1, 1, 1, 1, 1), 2, 3),
    (0, 3, 7, 5, 8, 3, 2, 12, (2, 0, 2, 1, 1, 1, 4), 1, 1),
    (1, 1, 9, 9, 6, 3, 3, 6, (2, 2, 1, 1, 2, 2, 6), 1, 1),
    (0, 2, 8, 8, 4, 1, 1, 4, (0, 0, 1, 1, 1, 1, 1), 2, 2),
])
def test_zero_point_decomposition_matches_direct_loop(case):
    kind, n, h, wd, c, r, s, k, prm, by, bx = case
    rng = np.random.default_rng(sum(case[:8]))
    lo, hi = (0, 255) if kind == 0 else (-128, 127)
    x = rng.integers(lo, hi + 1, size=(n, h, wd, c))
    G = prm[6]
    w = rng.integers(lo, hi + 1, size=(k * by * bx * r * s * (c // G),))
    zin = rng.integers(lo, hi + 1, size=n)
    zf = int(rng.integers(lo, hi + 1))
    got = _decomposed(x, w, zin, zf, n, h, wd, c, r, s, k, prm, by, bx)
    a = oracle.conv_args(n, h, wd, c, r, s, k, *prm, by, bx)
    want = oracle.conv_qi32(a, x.astype(np.float32), w.astype(np.float32), zin, zf)
    np.testing.assert_array_equal(got, want)
