"""Convolution entry points, mirroring the reference's conv interface (src/conv_types.h).

Reference-compatible (same names, argument meaning and errors):
  * ``Conv2DParams``, ``BlockConv2DParams``, ``ConvShape``, ``BlockConvShape``
    (src/conv_types.h:21-35, 112-123)
  * ``infer_conv_shape`` / ``infer_block_conv_shape`` (src/conv_types.h:125-169), raising
    ``RuntimeError`` with the reference's messages
  * ``launch_fprop_nhwc_qi32`` / ``launch_block_fprop_nhwc_qi32`` (src/conv_types.h:308-340):
    device pointers (torch CUDA tensors or integer addresses) to float codes, an int32 output,
    and device arrays of qparams; the qparams type selects LinQuantU8 / LinQuantS5.
New int8 path:
  * ``conv2d_s8`` -- int8 NHWC x int8 KRSC, int32 accumulation on tcgen05 tensor cores, fused
    bias / per-channel scale / round-half-even / clamp (ReLU, ReLU6) epilogue.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .quant import DataType, QPARAMS_TYPES, is_supported_quantized_input


# ctypes structs handed to the C ABI by pointer (it only reads them), one per distinct value.
_C_PARAMS: dict = {}
_C_EPILOGUES: dict = {}


@dataclass
class Conv2DParams:
    pad_h: int = 1
    pad_w: int = 1
    stride_h: int = 1
    stride_w: int = 1
    dilation_h: int = 1
    dilation_w: int = 1
    groups: int = 1

    def to_c(self) -> _lib.CConvParams:
        key = (self.pad_h, self.pad_w, self.stride_h, self.stride_w, self.dilation_h, self.dilation_w, self.groups)
        c = _C_PARAMS.get(key)
        if c is None:  # read-only use by the C ABI, so one struct per distinct value is shared
            c = _C_PARAMS[key] = _lib.CConvParams(*key)
        return c


@dataclass
class BlockConv2DParams:
    conv: Conv2DParams = None
    block_by: int = 1
    block_bx: int = 1

    def __post_init__(self):
        if self.conv is None:
            self.conv = Conv2DParams()


@dataclass
class ConvShape:
    ho: int = 0
    wo: int = 0
    cin_group: int = 0
    kout_group: int = 0


@dataclass
class BlockConvShape:
    base: ConvShape = None
    block_ho: int = 0
    block_wo: int = 0


def infer_conv_shape(x_shape, w_shape, p: Conv2DParams) -> ConvShape:
    """x_shape = (n, h, w, c); w_shape = (r, s, cin_per_group, k).  src/conv_types.h:125-146."""
    _, h, w, c = x_shape
    r, s, cin_per_group, k = w_shape
    if p.groups <= 0:
        raise RuntimeError("groups must be > 0")
    if c % p.groups != 0:
        raise RuntimeError("input channels must be divisible by groups")
    if k % p.groups != 0:
        raise RuntimeError("output channels must be divisible by groups")
    cin_group = c // p.groups
    if cin_group != cin_per_group:
        raise RuntimeError("filter cin_per_group mismatch")
    ho_num = h + 2 * p.pad_h - p.dilation_h * (r - 1) - 1
    wo_num = w + 2 * p.pad_w - p.dilation_w * (s - 1) - 1
    if ho_num < 0 or wo_num < 0:
        raise RuntimeError("invalid output size (negative numerator)")
    if p.stride_h <= 0 or p.stride_w <= 0:
        raise RuntimeError("stride must be > 0")
    ho = ho_num // p.stride_h + 1
    wo = wo_num // p.stride_w + 1
    if ho <= 0 or wo <= 0:
        raise RuntimeError("computed output size is <= 0")
    return ConvShape(ho, wo, cin_group, k // p.groups)


def infer_block_conv_shape(x_shape, w_block_shape, p: BlockConv2DParams) -> BlockConvShape:
    """w_block_shape = (k, by, bx, r, s, cin_per_group).  src/conv_types.h:148-169."""
    k, by, bx, r, s, cpg = w_block_shape
    if p.block_by <= 0 or p.block_bx <= 0:
        raise RuntimeError("block_by and block_bx must be > 0")
    if by != p.block_by or bx != p.block_bx:
        raise RuntimeError("blocked filter block grid mismatch")
    base = infer_conv_shape(x_shape, (r, s, cpg, k), p.conv)
    if base.ho % p.block_by != 0 or base.wo % p.block_bx != 0:
        raise RuntimeError("blocked convolution requires Ho/Wo divisible by block grid")
    return BlockConvShape(base, base.ho // p.block_by, base.wo // p.block_bx)


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if isinstance(t, torch.Tensor):
        if not t.is_cuda:
            raise RuntimeError("tensor arguments must be CUDA device tensors")
        return t.data_ptr()
    raise TypeError(f"expected a CUDA tensor or device address, got {type(t).__name__}")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(stream) -> int:
    """cudaStream_t of `stream`, or of the current device's current stream when None."""
    if stream is None:
        if _raw_stream is not None:  # the same handle as current_stream().cuda_stream, without the object
            return _raw_stream(torch.cuda.current_device())
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _qtype(qparams_type) -> DataType:
    if isinstance(qparams_type, DataType):
        dt = qparams_type
    else:
        dt = getattr(qparams_type, "dtype", None)
    if dt is None or not is_supported_quantized_input(dt):
        raise TypeError("launch_fprop_nhwc_qi32 supports only LinQuantU8 and LinQuantS5")
    return dt


def launch_fprop_nhwc_qi32(d_x, d_w, d_y, n, h, w, c, r, s, k, p: Conv2DParams, in_qp, f_qp,
                           qtype=DataType.LinQuantU8, stream=None) -> None:
    """Quantized conv fprop with int32 accumulators (src/conv_types.h:308-323).

    ``in_qp`` / ``f_qp``: device buffers holding QuantizationParameters structs of ``qtype``
    (see quant.qparams_to_device).
    """
    dt = _qtype(qtype)
    if in_qp is None or f_qp is None:
        raise RuntimeError("quantized CUDA fprop requires non-null quantization parameters")
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_fprop_nhwc_qi32(int(dt), _ptr(d_x), _ptr(d_w), _ptr(d_y), n, h, w, c, r, s, k,
                                                ctypes.byref(cp), _ptr(in_qp), _ptr(f_qp), _stream(stream)))


def launch_block_fprop_nhwc_qi32(d_x, d_w, d_y, n, h, w, c, r, s, k, p: BlockConv2DParams, in_qp, f_qp,
                                 qtype=DataType.LinQuantU8, stream=None) -> None:
    """Blocked quantized conv fprop (src/conv_types.h:325-340)."""
    dt = _qtype(qtype)
    if in_qp is None or f_qp is None:
        raise RuntimeError("quantized blocked CUDA fprop requires non-null quantization parameters")
    cp = p.conv.to_c()
    _lib.check(_lib.lib().b200q_block_fprop_nhwc_qi32(int(dt), _ptr(d_x), _ptr(d_w), _ptr(d_y), n, h, w, c, r, s,
                                                      k, ctypes.byref(cp), p.block_by, p.block_bx, _ptr(in_qp),
                                                      _ptr(f_qp), _stream(stream)))


@dataclass
class Epilogue:
    """Output stage of the int8 entry points (see include/b200q.h)."""

    out_kind: int = _lib.OUT_S8
    zp_out: int = 0
    clamp_lo: int = -128
    clamp_hi: int = 127

    @staticmethod
    def int32() -> "Epilogue":
        return Epilogue(_lib.OUT_S32, 0, 0, 0)

    @staticmethod
    def fp32() -> "Epilogue":
        return Epilogue(_lib.OUT_F32, 0, 0, 0)

    @staticmethod
    def int8(relu: bool = False, relu6_q: int | None = None, zp_out: int = 0) -> "Epilogue":
        lo = zp_out if (relu or relu6_q is not None) else -128
        hi = relu6_q if relu6_q is not None else 127
        return Epilogue(_lib.OUT_S8, zp_out, lo, hi)

    def to_c(self) -> _lib.CEpilogue:
        key = (self.out_kind, self.zp_out, self.clamp_lo, self.clamp_hi)
        c = _C_EPILOGUES.get(key)
        if c is None:
            c = _C_EPILOGUES[key] = _lib.CEpilogue(*key)
        return c

    @property
    def torch_dtype(self):
        return {_lib.OUT_S32: torch.int32, _lib.OUT_S8: torch.int8, _lib.OUT_F32: torch.float32}[self.out_kind]


def conv_out_shape(h, w, c, r, s, k, p: Conv2DParams):
    ho, wo = ctypes.c_int(), ctypes.c_int()
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv_out_shape(h, w, c, r, s, k, ctypes.byref(cp), ctypes.byref(ho), ctypes.byref(wo)))
    return ho.value, wo.value


def conv2d_s8_plan(n, h, w, c, r, s, k, p: Conv2DParams, epi: Epilogue, residual: bool = False) -> str:
    """Kernel family conv2d_s8 (conv2d_s8_add when residual) would use for this conv with 16-byte
    aligned tensors (a b200q_last_path name), decided on the host: no GPU needed."""
    path = ctypes.c_int()
    cp, ce = p.to_c(), epi.to_c()
    _lib.check(_lib.lib().b200q_conv2d_s8_plan(n, h, w, c, r, s, k, ctypes.byref(cp), ctypes.byref(ce), int(residual),
                                               ctypes.byref(path)))
    return _lib.PATH_NAMES.get(path.value, "?")


def conv2d_s8_into(y, x, w, bias, scale, n, h, wd, c, r, s, k, p: Conv2DParams, epi: Epilogue, stream=None) -> None:
    """Raw-pointer form: every tensor argument is a device tensor or address."""
    ce = epi.to_c()
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv2d_s8(_ptr(x), _ptr(w), _ptr(bias), _ptr(scale), _ptr(y), n, h, wd, c, r, s, k,
                                          ctypes.byref(cp), ctypes.byref(ce), _stream(stream)))


def conv2d_s8_add_into(y, x, w, bias, scale, res, res_scale: float, n, h, wd, c, r, s, k, p: Conv2DParams,
                       epi: Epilogue, stream=None) -> None:
    """conv2d_s8_into with a residual add fused into the int8 epilogue (b200q_conv2d_s8_add):
    p = fp32(acc + bias) * scale + fp32(res) * res_scale, rounded and clamped like Epilogue.int8."""
    ce = epi.to_c()
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv2d_s8_add(_ptr(x), _ptr(w), _ptr(bias), _ptr(scale), _ptr(res),
                                              ctypes.c_float(res_scale), _ptr(y), n, h, wd, c, r, s, k,
                                              ctypes.byref(cp), ctypes.byref(ce), _stream(stream)))


def conv2d_s8_add(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, scale: torch.Tensor,
                  res: torch.Tensor, res_scale: float, p: Conv2DParams, epi: Epilogue,
                  out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """int8 conv + residual: res is int8 with the output's shape [n, ho, wo, k]."""
    if x.dtype != torch.int8 or w.dtype != torch.int8 or res.dtype != torch.int8:
        raise TypeError("conv2d_s8_add takes int8 activations, weights and residual")
    n, h, wd, c = x.shape
    k, r, s, _ = w.shape
    ho, wo = conv_out_shape(h, wd, c, r, s, k, p)
    if tuple(res.shape) != (n, ho, wo, k):
        raise RuntimeError(f"residual shape {tuple(res.shape)} != output shape {(n, ho, wo, k)}")
    if out is None:
        out = torch.empty((n, ho, wo, k), dtype=torch.int8, device=x.device)
    conv2d_s8_add_into(out, x.contiguous(), w.contiguous(), bias, scale, res.contiguous(), res_scale, n, h, wd, c,
                       r, s, k, p, epi, stream)
    return out


def conv2d_s8(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, scale: torch.Tensor | None,
              p: Conv2DParams, epi: Epilogue, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """x: int8 [n,h,w,c]; w: int8 [k,r,s,c/groups]; bias int32 [k] or None; scale fp32 [k]."""
    if x.dtype != torch.int8 or w.dtype != torch.int8:
        raise TypeError("conv2d_s8 takes int8 activations and weights")
    n, h, wd, c = x.shape
    k, r, s, _ = w.shape
    ho, wo = conv_out_shape(h, wd, c, r, s, k, p)
    if out is None:
        out = torch.empty((n, ho, wo, k), dtype=epi.torch_dtype, device=x.device)
    conv2d_s8_into(out, x.contiguous(), w.contiguous(), bias, scale, n, h, wd, c, r, s, k, p, epi, stream)
    return out
