"""CPU check of the space-to-depth rewrite that the stem kernels implement (s2d_s8_kernel,
s2d_weight_s8_kernel and the tap-pair row tiles in my_own_cnn_b200/csrc): a stride-2 conv of a
1-4 channel input equals a stride-1 conv of the 2x2-block copy with the rearranged filter, whose
window starts floor(-pad / 2) blocks before each output position.  The index rules are restated
here in numpy, exactly as the kernels and the host dispatch compute them, and compared with the
C oracle's direct conv; the GPU parity tests check the kernels themselves."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.kat import rng_s8


def _fdiv2(v: int) -> int:
    return v // 2  # floor division, as the host's fdiv2


def _s2d_shape(r: int, s: int, pad_h: int, pad_w: int) -> tuple[int, int, int, int]:
    yoff, xoff = -((pad_h + 1) // 2), -((pad_w + 1) // 2)
    r2 = _fdiv2(r - 1 - pad_h) - yoff + 1
    s2 = (_fdiv2(s - 1 - pad_w) - xoff + 2) // 2 * 2
    return r2, s2, yoff, xoff


def _s2d_input(x: np.ndarray) -> np.ndarray:
    n, h, w, c = x.shape
    h2, w2 = (h + 1) // 2, (w + 1) // 2
    xs = np.zeros((n, h2, w2, 16), np.int64)
    for q in range(4):
        dy, dx = q >> 1, q & 1
        part = x[:, dy::2, dx::2, :]
        xs[:, : part.shape[1], : part.shape[2], q * c:(q + 1) * c] = part
    return xs


def _s2d_weights(wt: np.ndarray, r2: int, s2: int, pad_h: int, pad_w: int) -> np.ndarray:
    k, r, s, c = wt.shape
    yoff, xoff = -((pad_h + 1) // 2), -((pad_w + 1) // 2)
    ws = np.zeros((k, r2, s2, 16), np.int64)
    for R in range(r2):
        for S in range(s2):
            for cc in range(4 * c):
                q, ci = cc // c, cc % c
                rr = 2 * (R + yoff) + (q >> 1) + pad_h
                ss = 2 * (S + xoff) + (q & 1) + pad_w
                if 0 <= rr < r and 0 <= ss < s:
                    ws[:, R, S, cc] = wt[:, rr, ss, ci]
    return ws


@pytest.mark.parametrize("h,w,c,k,r,pad", [
    (64, 64, 3, 8, 7, 3),   # ResNet-50 stem: 4 x 4 taps
    (32, 32, 3, 8, 3, 1),   # MobileNetV2 stem: 2 x 2 taps
    (15, 17, 3, 4, 7, 3),   # odd H / W
    (9, 11, 1, 4, 3, 1),    # C = 1
    (10, 10, 4, 4, 5, 2),   # C = 4, even padding: 3 x 4 taps
    (13, 12, 2, 4, 3, 0),   # no padding
])
def test_space_to_depth_conv_equals_stride2_conv(h, w, c, k, r, pad):
    n = 2
    x = rng_s8(h * w + c, (n, h, w, c))
    wt = rng_s8(k * r + pad, (k, r, r, c))
    want = oracle.conv_s8(oracle.conv_args(n, h, w, c, r, r, k, pad, pad, 2, 2), x, wt)
    ho, wo = want.shape[1:3]
    r2, s2, yoff, xoff = _s2d_shape(r, r, pad, pad)
    assert 2 <= r2 <= 4 and s2 in (2, 4)
    xs, ws = _s2d_input(x), _s2d_weights(wt, r2, s2, pad, pad)
    # stride-1 conv of the block copy; window origin (ho + yoff, wo + xoff), zero outside
    big = np.zeros((n, xs.shape[1] + 16, xs.shape[2] + 16, 16), np.int64)
    big[:, 8:8 + xs.shape[1], 8:8 + xs.shape[2]] = xs
    got = np.zeros((n, ho, wo, k), np.int64)
    for R in range(r2):
        for S in range(s2):
            win = big[:, 8 + yoff + R:8 + yoff + R + ho, 8 + xoff + S:8 + xoff + S + wo, :]
            got += np.einsum("nhwc,kc->nhwk", win, ws[:, R, S, :])
    np.testing.assert_array_equal(got.astype(np.int32), want)


def test_row_tile_window_rows_cover_every_tap_read():
    """The window box holds ceil(((R2 - 1) * P + S2 - 1 + 128) / P) rows of P pixels: the last
    accumulator row of a tile reads pixel (R2 - 1) * P + (S2 - 1) + 127, inside the box."""
    for r2 in (2, 3, 4):
        for s2 in (2, 4):
            for wo in range(1, 128 - s2 + 2):
                p = wo + s2 - 1
                rows = ((r2 - 1) * p + s2 - 1 + 128 + p - 1) // p
                assert (r2 - 1) * p + (s2 - 1) + 127 < rows * p
                assert rows <= 256 and 2 * p <= 256  # TMA box limits (8-byte elements)
