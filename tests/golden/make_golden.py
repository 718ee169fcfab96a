"""Generate the golden known-answer fixtures in tests/golden/ (run in a container that has the reference).

Inputs follow the reference's own known-answer test, NikitaYak02/my_own_cnn quant_conv_test.cu:
  * codes   U8: (idx*37 + salt*19) % 251            (quant_conv_test.cu:20-23)
            S5: (idx*17 + salt*11) % 31 - 15        (quant_conv_test.cu:25-28)
  * input zero points per image  U8: 37 + 29*i,  S5: -5 + 7*i   (quant_conv_test.cu:40-60)
  * filter zero point            U8: 91,         S5: 3          (quant_conv_test.cu:65-81)
  * regular case: x 2x5x6x4, w 3x2x(4/2)x6, pad (1,0), groups 2  (quant_conv_test.cu:114-131)
  * blocked case: x 2x6x6x4, w 5x2x3x3x3x4, pad 1, block 2x3    (quant_conv_test.cu:163-182)
Outputs come from the reference's unmodified CPU oracle src/cpu_ref.cpp, compiled from its
sources into oracle/_ref/libref_oracle.so (oracle/Makefile).  Extra cases use the same code
formulas on other geometries (stride, dilation, groups, depthwise, C=3, K=1, N=1).

Usage:  python tests/golden/make_golden.py     (writes tests/golden/qconv_kat.npz)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle  # noqa: E402

U8, S5 = 0, 1


def codes(kind: int, count: int, salt: int) -> np.ndarray:
    idx = np.arange(count, dtype=np.int64)
    if kind == U8:
        v = (idx * 37 + salt * 19) % 251
    else:
        v = (idx * 17 + salt * 11) % 31 - 15
    return v.astype(np.float32)


def input_zps(kind: int, n: int) -> np.ndarray:
    i = np.arange(n)
    if kind == U8:
        return ((37 + 29 * i) % 256).astype(np.int32)  # uint8 wrap, as static_cast<uint8_t>
    return (((-5 + 7 * i) + 128) % 256 - 128).astype(np.int32)  # int8 wrap


def filter_zp(kind: int) -> int:
    return 91 if kind == U8 else 3


# name, kind, blocked, (n,h,w,c), (r,s,k), params(pad_h,pad_w,stride_h,stride_w,dil_h,dil_w,groups), (by,bx), salts
CASES = [
    ("regular_u8", U8, False, (2, 5, 6, 4), (3, 2, 6), (1, 0, 1, 1, 1, 1, 2), (1, 1), (1, 7)),
    ("regular_s5", S5, False, (2, 5, 6, 4), (3, 2, 6), (1, 0, 1, 1, 1, 1, 2), (1, 1), (1, 7)),
    ("blocked_u8", U8, True, (2, 6, 6, 4), (3, 3, 5), (1, 1, 1, 1, 1, 1, 1), (2, 3), (3, 9)),
    ("blocked_s5", S5, True, (2, 6, 6, 4), (3, 3, 5), (1, 1, 1, 1, 1, 1, 1), (2, 3), (3, 9)),
    ("stride2_u8", U8, False, (2, 9, 7, 8), (3, 3, 5), (1, 1, 2, 2, 1, 1, 1), (1, 1), (2, 5)),
    ("dilation2_s5", S5, False, (1, 8, 9, 6), (3, 3, 4), (2, 2, 1, 1, 2, 2, 1), (1, 1), (4, 6)),
    ("groups4_u8", U8, False, (3, 6, 5, 8), (3, 3, 12), (1, 1, 1, 1, 1, 1, 4), (1, 1), (5, 8)),
    ("depthwise_s5", S5, False, (2, 7, 7, 6), (3, 3, 6), (1, 1, 2, 1, 1, 1, 6), (1, 1), (6, 2)),
    ("stem_c3_u8", U8, False, (1, 12, 12, 3), (7, 7, 4), (3, 3, 2, 2, 1, 1, 1), (1, 1), (7, 3)),
    ("k1_n1_s5", S5, False, (1, 4, 4, 5), (1, 1, 1), (0, 0, 1, 1, 1, 1, 1), (1, 1), (8, 4)),
    ("blocked_groups2_s5", S5, True, (2, 4, 6, 4), (3, 3, 4), (1, 1, 1, 1, 1, 1, 2), (2, 2), (9, 1)),
    ("asym_pad_u8", U8, False, (2, 5, 7, 3), (2, 4, 5), (0, 2, 1, 3, 1, 1, 1), (1, 1), (10, 11)),
]


def build_case(name, kind, blocked, xs, rsk, prm, blk, salts):
    n, h, w, c = xs
    r, s, k = rsk
    pad_h, pad_w, sh, sw, dh, dw, groups = prm
    by, bx = blk
    cpg = c // groups
    x = codes(kind, n * h * w * c, salts[0]).reshape(n, h, w, c)
    wcount = k * by * bx * r * s * cpg if blocked else k * r * s * cpg
    wt = codes(kind, wcount, salts[1])
    a = oracle.conv_args(n, h, w, c, r, s, k, pad_h, pad_w, sh, sw, dh, dw, groups, by, bx)
    zin = input_zps(kind, n)
    zf = filter_zp(kind)
    y = oracle.ref_conv_qi32(a, kind, x, wt, zin, zf, blocked)
    return {
        f"{name}/x": x, f"{name}/w": wt, f"{name}/zp_in": zin, f"{name}/zp_f": np.int32(zf),
        f"{name}/y": y, f"{name}/meta": np.array([kind, int(blocked), n, h, w, c, r, s, k, pad_h, pad_w, sh, sw,
                                                 dh, dw, groups, by, bx], dtype=np.int32),
    }


def main() -> None:
    if not oracle.ref_available():
        raise SystemExit("oracle/_ref/libref_oracle.so missing: run `make -C oracle` with the reference present")
    arrays = {}
    for case in CASES:
        arrays.update(build_case(*case))
    arrays["names"] = np.array([c[0] for c in CASES])
    out = Path(__file__).resolve().parent / "qconv_kat.npz"
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({len(CASES)} cases)")


if __name__ == "__main__":
    main()
