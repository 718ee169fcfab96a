"""ctypes front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may use this
module, and only as the checker or the timed CPU baseline.  Nothing in my_own_cnn_b200 imports it.

Two oracles:
  * ``liboracle.so``          -- oracle.c, a C restatement of the reference algorithms
                                 (src/cpu_ref.cpp:36-112, bmm.h:9-29) plus the new requant epilogue;
  * ``_ref/libref_oracle.so`` -- the reference's own src/cpu_ref.cpp compiled from its sources
                                 (built in a container that has the reference; travels prebuilt).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, Structure, c_float, c_int, c_int8, c_int32, c_size_t, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_oracle.so"


class ConvArgs(Structure):
    """orc_conv_t (oracle.c) == Args (ref_capi.cpp)."""

    _fields_ = [(f, c_int) for f in ("n", "h", "w", "c", "r", "s", "k", "pad_h", "pad_w", "stride_h", "stride_w",
                                     "dil_h", "dil_w", "groups", "by", "bx")]


def conv_args(n, h, w, c, r, s, k, pad_h=1, pad_w=1, stride_h=1, stride_w=1, dil_h=1, dil_w=1, groups=1, by=1, bx=1):
    return ConvArgs(n, h, w, c, r, s, k, pad_h, pad_w, stride_h, stride_w, dil_h, dil_w, groups, by, bx)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
        L = ctypes.CDLL(str(LIB))
        vp = c_void_p
        L.orc_conv_out_shape.argtypes = [c_int] * 13 + [POINTER(c_int), POINTER(c_int)]
        L.orc_conv_qi32.argtypes = [POINTER(ConvArgs), vp, vp, vp, vp, c_int32]
        L.orc_conv_s8.argtypes = [POINTER(ConvArgs), vp, vp, vp, c_int]
        L.orc_requant_s8.argtypes = [vp, c_size_t, c_int, vp, vp, c_int, c_int, c_int, vp]
        L.orc_requant_s8.restype = None
        L.orc_dequant_f32.argtypes = [vp, c_size_t, c_int, vp, vp, vp]
        L.orc_requant_res_s8.argtypes = [vp, c_size_t, c_int, vp, vp, vp, c_float, c_int, c_int, c_int, vp]
        L.orc_maxpool_s8.argtypes = [vp, vp] + [c_int] * 10
        L.orc_global_avgpool_s8.argtypes = [vp, vp] + [c_int] * 4
        L.orc_dequant_f32.restype = None
        L.orc_bmm_i32.argtypes = [vp, vp, vp] + [c_int] * 6
        L.orc_bmm_i32.restype = None
        L.orc_bmm_s8.argtypes = [vp, vp, vp] + [c_int] * 7
        L.orc_bmm_s8.restype = None
        L.orc_fill_s8_uniform.argtypes = [c_uint64, c_uint64, c_int, c_int, c_size_t, c_size_t, vp]
        L.orc_fill_s8_uniform.restype = None
        L.orc_fill_i32_uniform.argtypes = [c_uint64, c_uint64, c_int32, c_int32, c_size_t, c_size_t, vp]
        L.orc_fill_i32_uniform.restype = None
        L.orc_fill_s8_table.argtypes = [c_uint64, c_uint64, vp, c_size_t, c_size_t, vp]
        L.orc_fill_s8_table.restype = None
        L.orc_fill_f32_uniform.argtypes = [c_uint64, c_uint64, c_float, c_float, c_size_t, c_size_t, vp]
        L.orc_fill_f32_uniform.restype = None
        _lib = L
    return _lib


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError("oracle/_ref/libref_oracle.so is not built (needs the reference sources)")
        L = ctypes.CDLL(str(REF_LIB))
        vp = c_void_p
        L.ref_fprop_qi32.argtypes = [POINTER(ConvArgs), c_int, c_int, vp, vp, vp, vp, c_int32]
        L.ref_fprop_qi32_threaded.argtypes = [POINTER(ConvArgs), c_int, vp, vp, vp, vp, c_int32, c_int]
        _ref = L
    return _ref


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def out_shape(a: ConvArgs):
    ho, wo = c_int(), c_int()
    rc = lib().orc_conv_out_shape(a.h, a.w, a.c, a.r, a.s, a.k, a.pad_h, a.pad_w, a.stride_h, a.stride_w, a.dil_h,
                                  a.dil_w, a.groups, ctypes.byref(ho), ctypes.byref(wo))
    if rc:
        raise RuntimeError("invalid conv shape")
    return ho.value, wo.value


def conv_qi32(a: ConvArgs, x: np.ndarray, w: np.ndarray, zp_in, zp_f: int) -> np.ndarray:
    """Restated reference conv (float codes, zero points) -> int32 [n, ho, wo, k]."""
    ho, wo = out_shape(a)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    zp = np.ascontiguousarray(zp_in, dtype=np.int32)
    y = np.zeros((a.n, ho, wo, a.k), dtype=np.int32)
    if lib().orc_conv_qi32(ctypes.byref(a), _p(x), _p(w), _p(y), _p(zp), int(zp_f)):
        raise RuntimeError("invalid conv shape")
    return y


def ref_conv_qi32(a: ConvArgs, kind: int, x: np.ndarray, w: np.ndarray, zp_in, zp_f: int, blocked: bool) -> np.ndarray:
    """The reference's own cpu_fprop_nhwc_qi32 / cpu_block_fprop_nhwc_qi32 (kind 0 = U8, 1 = S5)."""
    ho, wo = out_shape(a)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    zp = np.ascontiguousarray(zp_in, dtype=np.int32)
    y = np.zeros((a.n, ho, wo, a.k), dtype=np.int32)
    if ref_lib().ref_fprop_qi32(ctypes.byref(a), kind, int(blocked), _p(x), _p(w), _p(y), _p(zp), int(zp_f)):
        raise RuntimeError("reference rejected the shape")
    return y


def ref_conv_qi32_threaded(a: ConvArgs, x: np.ndarray, w: np.ndarray, threads: int) -> np.ndarray:
    """Reference cpu_fprop_nhwc_qi32 (S5 qparams, zero points 0) over image slices on `threads` threads."""
    ho, wo = out_shape(a)
    zp = np.zeros(a.n, dtype=np.int32)
    y = np.empty((a.n, ho, wo, a.k), dtype=np.int32)
    if ref_lib().ref_fprop_qi32_threaded(ctypes.byref(a), 1, _p(x), _p(w), _p(y), _p(zp), 0, threads):
        raise RuntimeError("reference rejected the shape")
    return y


def conv_s8(a: ConvArgs, x: np.ndarray, w: np.ndarray, threads: int = 1) -> np.ndarray:
    """int8 conv, zero points 0 -> int32 accumulators [n, ho, wo, k]."""
    ho, wo = out_shape(a)
    x = np.ascontiguousarray(x, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    y = np.empty((a.n, ho, wo, a.k), dtype=np.int32)
    if lib().orc_conv_s8(ctypes.byref(a), _p(x), _p(w), _p(y), threads):
        raise RuntimeError("invalid conv shape")
    return y


def requant_s8(acc: np.ndarray, bias, scale: np.ndarray, zp: int = 0, lo: int = -128, hi: int = 127) -> np.ndarray:
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    k = acc.shape[-1]
    rows = acc.size // k
    sc = np.ascontiguousarray(scale, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.int32)
    out = np.empty(acc.shape, dtype=np.int8)
    lib().orc_requant_s8(_p(acc), rows, k, None if b is None else _p(b), _p(sc), zp, lo, hi, _p(out))
    return out


def requant_res_s8(acc: np.ndarray, bias, scale: np.ndarray, res: np.ndarray, res_scale: float, zp: int = 0,
                   lo: int = -128, hi: int = 127) -> np.ndarray:
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    k = acc.shape[-1]
    sc = np.ascontiguousarray(scale, dtype=np.float32)
    rs = np.ascontiguousarray(res, dtype=np.int8)
    assert rs.size == acc.size
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.int32)
    out = np.empty(acc.shape, dtype=np.int8)
    lib().orc_requant_res_s8(_p(acc), acc.size // k, k, None if b is None else _p(b), _p(sc), _p(rs),
                             float(res_scale), zp, lo, hi, _p(out))
    return out


def maxpool_s8(x: np.ndarray, r: int, s: int, stride_h: int, stride_w: int, pad_h: int, pad_w: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int8)
    n, h, w, c = x.shape
    ho, wo = (h + 2 * pad_h - r) // stride_h + 1, (w + 2 * pad_w - s) // stride_w + 1
    y = np.empty((n, ho, wo, c), dtype=np.int8)
    if lib().orc_maxpool_s8(_p(x), _p(y), n, h, w, c, r, s, stride_h, stride_w, pad_h, pad_w):
        raise RuntimeError("invalid pool shape")
    return y


def global_avgpool_s8(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int8)
    n, h, w, c = x.shape
    y = np.empty((n, c), dtype=np.int8)
    lib().orc_global_avgpool_s8(_p(x), _p(y), n, h, w, c)
    return y


def dequant_f32(acc: np.ndarray, bias, scale: np.ndarray) -> np.ndarray:
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    k = acc.shape[-1]
    sc = np.ascontiguousarray(scale, dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.int32)
    out = np.empty(acc.shape, dtype=np.float32)
    lib().orc_dequant_f32(_p(acc), acc.size // k, k, None if b is None else _p(b), _p(sc), _p(out))
    return out


def bias_add_i32(acc: np.ndarray, bias) -> np.ndarray:
    """acc + bias with int32 wrap-around (the S32 epilogue)."""
    if bias is None:
        return np.asarray(acc, dtype=np.int32)
    s = np.asarray(acc, dtype=np.int64) + np.asarray(bias, dtype=np.int64)
    return ((s + 2**31) % 2**32 - 2**31).astype(np.int32)


def bmm_i32(A, B, batch, M, N, K, ta, tb) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.int32)
    B = np.ascontiguousarray(B, dtype=np.int32)
    C = np.empty((batch, M, N), dtype=np.int32)
    lib().orc_bmm_i32(_p(A), _p(B), _p(C), batch, M, N, K, int(ta), int(tb))
    return C


def bmm_s8(A, B, batch, M, N, K, ta, tb, threads: int = 1) -> np.ndarray:
    A = np.ascontiguousarray(A, dtype=np.int8)
    B = np.ascontiguousarray(B, dtype=np.int8)
    C = np.empty((batch, M, N), dtype=np.int32)
    lib().orc_bmm_s8(_p(A), _p(B), _p(C), batch, M, N, K, int(ta), int(tb), threads)
    return C


def fill_s8_uniform(seed, tensor_id, lo, hi, offset, count) -> np.ndarray:
    out = np.empty(count, dtype=np.int8)
    lib().orc_fill_s8_uniform(seed, tensor_id, lo, hi, offset, count, _p(out))
    return out


def fill_i32_uniform(seed, tensor_id, lo, hi, offset, count) -> np.ndarray:
    out = np.empty(count, dtype=np.int32)
    lib().orc_fill_i32_uniform(seed, tensor_id, lo, hi, offset, count, _p(out))
    return out


def fill_s8_table(seed, tensor_id, table: np.ndarray, offset, count) -> np.ndarray:
    t = np.ascontiguousarray(table, dtype=np.int8)
    out = np.empty(count, dtype=np.int8)
    lib().orc_fill_s8_table(seed, tensor_id, _p(t), offset, count, _p(out))
    return out


def fill_f32_uniform(seed, tensor_id, lo, hi, offset, count) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().orc_fill_f32_uniform(seed, tensor_id, lo, hi, offset, count, _p(out))
    return out


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def ref_conv_f32(a: ConvArgs, op: int, blocked: bool, in_a: np.ndarray, in_b: np.ndarray, out_shape,
                 bias: np.ndarray | None = None, bias_mode: int = 0) -> np.ndarray:
    """The reference's own fp32 CPU loops (src/cpu_ref.cpp:116-371): op 0 fprop (x, w) -> y,
    1 bprop (dy, w) -> dx, 2 grad (x, dy) -> dw.  For blocked grad, `bias` receives dbias."""
    in_a = np.ascontiguousarray(in_a, dtype=np.float32)
    in_b = np.ascontiguousarray(in_b, dtype=np.float32)
    out = np.zeros(out_shape, dtype=np.float32)
    bptr = None if bias is None else _p(bias)
    lib_ = ref_lib()
    lib_.ref_conv_f32.argtypes = [ctypes.c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int]
    if lib_.ref_conv_f32(ctypes.byref(a), op, int(blocked), _p(in_a), _p(in_b), _p(out), bptr, bias_mode):
        raise RuntimeError("reference rejected the shape")
    return out
