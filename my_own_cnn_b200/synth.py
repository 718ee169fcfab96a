"""Seeded synthetic tensors, generated on the GPU by a counter-based splitmix64 stream.

Element i of tensor (seed, tensor_id) depends only on (seed, tensor_id, i), so any slice (one
image, one GPU's shard) can be regenerated independently -- by the CPU oracle too.
Normal / half-normal int8 codes come from a 65536-entry quantile table computed here on the
host (the table is the distribution; the device only indexes it, so CPU and GPU agree exactly).
"""
from __future__ import annotations

from functools import lru_cache
from statistics import NormalDist

import numpy as np
import torch

from . import _lib
from .conv import _stream


def quantile_table(kind: str, sigma: float, lo: int, hi: int) -> np.ndarray:
    """int8 codes: table[u] = clip(rint(q((u + 0.5) / 65536)), lo, hi).

    kind 'normal': q = sigma * Phi^-1(p); 'halfnormal': q = sigma * Phi^-1((1 + p) / 2)."""
    return _quantile_table(kind, float(sigma), int(lo), int(hi)).copy()


@lru_cache(maxsize=None)
def _quantile_table(kind: str, sigma: float, lo: int, hi: int) -> np.ndarray:
    nd = NormalDist(0.0, sigma)
    out = np.empty(65536, dtype=np.int8)
    for u in range(65536):
        p = (u + 0.5) / 65536.0
        if kind == "halfnormal":
            p = (1.0 + p) / 2.0
        elif kind != "normal":
            raise ValueError(kind)
        out[u] = int(np.clip(np.rint(nd.inv_cdf(p)), lo, hi))
    return out


def fill_s8_uniform(t: torch.Tensor, seed: int, tensor_id: int, lo: int = -127, hi: int = 127, stream=None):
    assert t.dtype == torch.int8 and t.is_cuda and t.is_contiguous()
    _lib.check(_lib.lib().b200q_fill_s8_uniform(t.data_ptr(), t.numel(), seed, tensor_id, lo, hi, _stream(stream)))
    return t


def fill_i32_uniform(t: torch.Tensor, seed: int, tensor_id: int, lo: int, hi: int, stream=None):
    assert t.dtype == torch.int32 and t.is_cuda and t.is_contiguous()
    _lib.check(_lib.lib().b200q_fill_i32_uniform(t.data_ptr(), t.numel(), seed, tensor_id, lo, hi, _stream(stream)))
    return t


def fill_s8_table(t: torch.Tensor, seed: int, tensor_id: int, table: torch.Tensor, stream=None):
    assert t.dtype == torch.int8 and t.is_cuda and table.is_cuda and table.numel() == 65536
    _lib.check(_lib.lib().b200q_fill_s8_table(t.data_ptr(), t.numel(), seed, tensor_id, table.data_ptr(),
                                              _stream(stream)))
    return t


def scales_f32(n: int, seed: int, tensor_id: int, lo: float = 1e-4, hi: float = 1e-3) -> np.ndarray:
    """Per-channel requant scales U[lo, hi), fp32, generated on the host (same splitmix64 stream)."""
    key = stream_key(seed, tensor_id)
    i = np.arange(n, dtype=np.uint64)
    u = (draw(key, i) >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    return (np.float32(lo) + u * (np.float32(hi) - np.float32(lo))).astype(np.float32)


_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_G = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def stream_key(seed: int, tensor_id: int) -> np.uint64:
    with np.errstate(over="ignore"):
        return _mix64(np.uint64(seed) * _G ^ _mix64(np.uint64(tensor_id) + np.uint64(0x632BE59BD9B4E019)))


def draw(key, i):
    with np.errstate(over="ignore"):
        return _mix64(np.uint64(key) + (np.asarray(i, dtype=np.uint64) + np.uint64(1)) * _G)


def s8_uniform_host(seed: int, tensor_id: int, lo: int, hi: int, offset: int, count: int) -> np.ndarray:
    """Host copy of elements [offset, offset+count) of fill_s8_uniform."""
    key = stream_key(seed, tensor_id)
    u = draw(key, np.arange(offset, offset + count, dtype=np.uint64)) >> np.uint64(32)
    span = np.uint64(hi - lo + 1)
    return (lo + ((u * span) >> np.uint64(32)).astype(np.int64)).astype(np.int8)


def i32_uniform_host(seed: int, tensor_id: int, lo: int, hi: int, offset: int, count: int) -> np.ndarray:
    key = stream_key(seed, tensor_id)
    u = draw(key, np.arange(offset, offset + count, dtype=np.uint64)) >> np.uint64(32)
    span = np.uint64(hi - lo + 1)
    with np.errstate(over="ignore"):
        return (lo + ((u * span) >> np.uint64(32)).astype(np.int64)).astype(np.int32)


def s8_table_host(seed: int, tensor_id: int, table: np.ndarray, offset: int, count: int) -> np.ndarray:
    key = stream_key(seed, tensor_id)
    idx = draw(key, np.arange(offset, offset + count, dtype=np.uint64)) >> np.uint64(48)
    return table[idx.astype(np.int64)]
