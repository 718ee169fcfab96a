"""Quantization types of the reference (src/nnalgebra_quantization.h), mirrored for Python callers.

The ctypes structures have the exact memory layout of the C++ structs, so an array of them
copied to the device is what the reference's launchers receive as ``in_qp`` / ``f_qp``.
Only ``zero_point`` is read by any reference computation (getZeroPoint, :56-81).
"""
from __future__ import annotations

import ctypes
from enum import IntEnum

import torch


class DataType(IntEnum):
    """src/nnalgebra_quantization.h:19-24."""

    Real32 = 0
    LinQuantU8 = 1
    LinQuantS5 = 2
    LinQuantI32 = 3


class QuantizationParametersU8(ctypes.Structure):
    """QuantizationParameters<LinQuantU8> (src/nnalgebra_quantization.h:29-34)."""

    _fields_ = [("zero_point", ctypes.c_uint8), ("scale", ctypes.c_float), ("symmetric", ctypes.c_bool)]
    dtype = DataType.LinQuantU8

    def __init__(self, zero_point: int = 0, scale: float = 1.0, symmetric: bool = False):
        super().__init__(zero_point, scale, symmetric)


class QuantizationParametersS5(ctypes.Structure):
    """QuantizationParameters<LinQuantS5> (src/nnalgebra_quantization.h:36-41)."""

    _fields_ = [("zero_point", ctypes.c_int8), ("n_bins", ctypes.c_uint8), ("scale", ctypes.c_float)]
    dtype = DataType.LinQuantS5

    def __init__(self, zero_point: int = 0, n_bins: int = 0, scale: float = 1.0):
        super().__init__(zero_point, n_bins, scale)


QPARAMS_TYPES = {DataType.LinQuantU8: QuantizationParametersU8, DataType.LinQuantS5: QuantizationParametersS5}


def get_zero_point(qp) -> int:
    """getZeroPoint (src/nnalgebra_quantization.h:56-81)."""
    if isinstance(qp, (QuantizationParametersU8, QuantizationParametersS5)):
        return int(qp.zero_point)
    raise TypeError(f"unsupported quantization parameters {type(qp).__name__}")


def is_supported_quantized_input(dtype: DataType) -> bool:
    """kIsSupportedQuantizedInput (src/nnalgebra_quantization.h:83-93)."""
    return dtype in (DataType.LinQuantU8, DataType.LinQuantS5)


def qparams_to_device(qps, device="cuda") -> torch.Tensor:
    """Copy a sequence of qparams structs (one type) to device memory as raw bytes.

    The returned uint8 tensor's data pointer is what ``in_qp`` / ``f_qp`` expect.
    """
    qps = list(qps) if not isinstance(qps, ctypes.Structure) else [qps]
    if not qps:
        raise ValueError("empty qparams list")
    t = type(qps[0])
    if any(type(q) is not t for q in qps):
        raise TypeError("mixed qparams types")
    arr = (t * len(qps))(*qps)
    raw = bytes(arr)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)
