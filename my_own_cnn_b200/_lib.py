"""ctypes binding of libb200q.so (the C ABI in include/b200q.h).

The library is loaded from the package directory.  There is no fallback: if the shared
library is missing or fails to load, importing an op raises, so a GPU run can never silently
use anything but the CUDA kernels.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_int, c_int8, c_int32, c_int64, c_longlong, c_size_t, c_uint8
from ctypes import c_uint64, c_void_p, c_float, c_char_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200q.so"

B200Q_OK = 0
B200Q_ERR_INVALID_ARG = 1
B200Q_ERR_UNSUPPORTED = 2
B200Q_ERR_CUDA = 3
B200Q_ERR_TIMEOUT = 4

OUT_S32, OUT_S8, OUT_F32 = 0, 1, 2

PATH_NAMES = {
    0: "none",
    1: "tcgen05-im2col",
    2: "tcgen05-tiled",
    3: "cuda-core-generic",
    4: "cuda-core-depthwise",
    5: "cuda-core-qi32",
    6: "cuda-core-bmm-i32",
    7: "tcgen05-packed",
    8: "tcgen05-tiled-2sm",
    9: "tcgen05-rowtile",
    10: "tcgen05-s2d",
    11: "tcgen05-qi32",
    12: "cuda-core-depthwise-tma",
    13: "tcgen05-f32",
    14: "cuda-core-f32",
    15: "tcgen05-tiled-grouped",
    16: "tcgen05-bmm-i32",
}


class CConvParams(Structure):
    """Same layout as Conv2DParams (src/conv_types.h:21-29)."""

    _fields_ = [("pad_h", c_int), ("pad_w", c_int), ("stride_h", c_int), ("stride_w", c_int),
                ("dilation_h", c_int), ("dilation_w", c_int), ("groups", c_int)]


class CEpilogue(Structure):
    _fields_ = [("out_kind", c_int), ("zp_out", c_int), ("clamp_lo", c_int), ("clamp_hi", c_int)]


class B200QError(RuntimeError):
    """Raised for a non-zero status; ``code`` is the b200q_status value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                           "(the CUDA library is required, there is no CPU path)")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, i = c_void_p, c_int
    pconv, pepi = POINTER(CConvParams), POINTER(CEpilogue)
    sig = {
        "b200q_fprop_nhwc_qi32": [i, vp, vp, vp, i, i, i, i, i, i, i, pconv, vp, vp, vp],
        "b200q_block_fprop_nhwc_qi32": [i, vp, vp, vp, i, i, i, i, i, i, i, pconv, i, i, vp, vp, vp],
        "b200q_bmm_matmul_i32": [vp, vp, vp, i, i, i, i, i, i, vp],
        "b200q_conv2d_s8": [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, pconv, pepi, vp],
        "b200q_conv2d_s8_packed_noalloc": [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, pconv, pepi, vp],
        "b200q_conv2d_s8_add": [vp, vp, vp, vp, vp, c_float, vp, i, i, i, i, i, i, i, pconv, pepi, vp],
        "b200q_maxpool_s8": [vp, vp, i, i, i, i, i, i, i, i, i, i, vp],
        "b200q_global_avgpool_s8": [vp, vp, i, i, i, i, vp],
        "b200q_bmm_s8": [vp, vp, vp, vp, vp, i, i, i, i, i, i, pepi, vp],
        "b200q_conv_out_shape": [i, i, i, i, i, i, pconv, POINTER(c_int), POINTER(c_int)],
        "b200q_conv2d_s8_plan": [i, i, i, i, i, i, i, pconv, pepi, i, POINTER(c_int)],
        "b200q_device_error": [],
        "b200q_last_path": [],
        "b200q_fill_s8_uniform": [vp, c_size_t, c_uint64, c_uint64, i, i, vp],
        "b200q_fill_i32_uniform": [vp, c_size_t, c_uint64, c_uint64, c_int32, c_int32, vp],
        "b200q_fill_s8_table": [vp, c_size_t, c_uint64, c_uint64, vp, vp],
        "b200q_selftest_wait_timeout": [c_longlong],
        "b200q_conv_fprop_f32": [vp, vp, vp, i, vp, i, i, i, i, i, i, i, pconv, i, i, vp],
        "b200q_conv_bprop_f32": [vp, vp, vp, i, i, i, i, i, i, i, pconv, i, i, vp],
        "b200q_conv_grad_f32": [vp, vp, vp, vp, i, i, i, i, i, i, i, i, pconv, i, i, vp],
        "b200q_bmm_f32": [vp, vp, vp, i, i, i, i, i, i, vp],
    }
    for name, args in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = c_int
    L.b200q_last_error.argtypes = []
    L.b200q_last_error.restype = c_char_p
    L.b200q_set_path_policy.argtypes = [c_int]
    L.b200q_set_path_policy.restype = None
    L.b200q_noalloc_scratch_bytes.argtypes = []
    L.b200q_noalloc_scratch_bytes.restype = c_size_t
    L.b200q_tc_launch_count.argtypes = []
    L.b200q_tc_launch_count.restype = c_longlong
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != B200Q_OK:
        msg = lib().b200q_last_error().decode(errors="replace")
        raise B200QError(rc, msg)


def last_path() -> str:
    return PATH_NAMES.get(lib().b200q_last_path(), "?")


def set_path_policy(policy: int) -> None:
    lib().b200q_set_path_policy(policy)


def tc_launch_count() -> int:
    return int(lib().b200q_tc_launch_count())


EXPORTED_SYMBOLS = [
    "b200q_fprop_nhwc_qi32", "b200q_block_fprop_nhwc_qi32", "b200q_bmm_matmul_i32",
    "b200q_conv2d_s8", "b200q_bmm_s8", "b200q_conv_out_shape", "b200q_last_error",
    "b200q_device_error", "b200q_last_path", "b200q_set_path_policy", "b200q_tc_launch_count",
    "b200q_fill_s8_uniform", "b200q_fill_i32_uniform", "b200q_fill_s8_table",
    "b200q_selftest_wait_timeout", "b200q_conv2d_s8_packed_noalloc", "b200q_noalloc_scratch_bytes",
    "b200q_conv_fprop_f32", "b200q_conv_bprop_f32", "b200q_conv_grad_f32", "b200q_bmm_f32",
    "b200q_conv2d_s8_add", "b200q_maxpool_s8", "b200q_global_avgpool_s8", "b200q_conv2d_s8_plan",
]
