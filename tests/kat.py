"""Helpers shared by the tests: golden-case decoding and seeded host data."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class KatCase:
    name: str
    kind: int  # 0 = LinQuantU8, 1 = LinQuantS5
    blocked: bool
    n: int
    h: int
    w: int
    c: int
    r: int
    s: int
    k: int
    pad_h: int
    pad_w: int
    stride_h: int
    stride_w: int
    dil_h: int
    dil_w: int
    groups: int
    by: int
    bx: int
    x: np.ndarray
    wt: np.ndarray
    zp_in: np.ndarray
    zp_f: int
    y: np.ndarray


def kat_cases(golden) -> list[KatCase]:
    out = []
    for name in golden["names"]:
        name = str(name)
        m = [int(v) for v in golden[f"{name}/meta"]]
        out.append(KatCase(name, m[0], bool(m[1]), *m[2:18], golden[f"{name}/x"], golden[f"{name}/w"],
                           golden[f"{name}/zp_in"], int(golden[f"{name}/zp_f"]), golden[f"{name}/y"]))
    return out


def rng_s8(seed: int, shape, lo: int = -127, hi: int = 127) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=shape, dtype=np.int64).astype(np.int8)
