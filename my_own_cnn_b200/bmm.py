"""Batched GEMM entry points, mirroring the reference's bmm API (bmm.h).

  * ``bmm_matmul_i32(A, B, C, batch, M, N, K, trans_a, trans_b)`` -- bmm.h:69-74, int32 inputs,
    int32 wrap-around results; layouts as bmm.h:9-29.
  * ``bmm_s8`` -- int8 inputs on tcgen05 tensor cores, int32 accumulation, per-column
    bias / scale epilogue (int32, int8-requantized or fp32 outputs).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .conv import Epilogue, _ptr, _stream

BMM_TRANSPOSE_NONE = 0
BMM_TRANSPOSE_YES = 1


def bmm_matmul_i32(A, B, C, batch, M, N, K, trans_a=BMM_TRANSPOSE_NONE, trans_b=BMM_TRANSPOSE_NONE,
                   stream=None) -> None:
    _lib.check(_lib.lib().b200q_bmm_matmul_i32(_ptr(A), _ptr(B), _ptr(C), batch, M, N, K, int(trans_a),
                                               int(trans_b), _stream(stream)))


def bmm_s8_into(C, A, B, bias, col_scale, batch, M, N, K, trans_a, trans_b, epi: Epilogue, stream=None) -> None:
    ce = epi.to_c()
    _lib.check(_lib.lib().b200q_bmm_s8(_ptr(A), _ptr(B), _ptr(bias), _ptr(col_scale), _ptr(C), batch, M, N, K,
                                       int(trans_a), int(trans_b), ctypes.byref(ce), _stream(stream)))


def bmm_s8(A: torch.Tensor, B: torch.Tensor, trans_a: int = 0, trans_b: int = 0, epi: Epilogue | None = None,
           bias: torch.Tensor | None = None, col_scale: torch.Tensor | None = None,
           out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """A: [batch, M, K] (or [batch, K, M] with trans_a); B: [batch, K, N] (or [batch, N, K] with trans_b)."""
    if A.dtype != torch.int8 or B.dtype != torch.int8:
        raise TypeError("bmm_s8 takes int8 operands")
    epi = epi or Epilogue.int32()
    batch = A.shape[0]
    M, K = (A.shape[2], A.shape[1]) if trans_a else (A.shape[1], A.shape[2])
    N = B.shape[1] if trans_b else B.shape[2]
    if out is None:
        out = torch.empty((batch, M, N), dtype=epi.torch_dtype, device=A.device)
    bmm_s8_into(out, A.contiguous(), B.contiguous(), bias, col_scale, batch, M, N, K, trans_a, trans_b, epi, stream)
    return out
