"""fp32 entry points, mirroring the reference's fp32 conv and bmm interfaces.

  * ``launch_fprop_nhwc / launch_bprop_nhwc / launch_grad_nhwc`` (src/conv_types.h:287-295) and the
    blocked ``launch_block_{fprop,bprop,grad}_nhwc`` with their bias arguments
    (src/conv_types.h:296-306, BlockBiasMode src/conv_types.h:36-39);
  * ``bmm_matmul`` and the bmm layer API ``bmm_fprop / bmm_bprop_dA / bmm_bprop_dB / bmm_bprop``
    (bmm.h:36-66, defined over bmm_matmul as bmm.cu:324-361 does).
Arguments are device tensors (torch CUDA tensors or integer addresses) in the reference's layouts;
invalid shapes raise RuntimeError with the reference's messages.  The work runs on tcgen05 tensor
cores with 3 x TF32 split products (see include/b200q.h).
"""
from __future__ import annotations

import ctypes
import enum

from . import _lib
from .conv import BlockConv2DParams, Conv2DParams, _ptr, _stream


class BlockBiasMode(enum.IntEnum):
    PerBlock = 0
    Shared = 1


def launch_fprop_nhwc(d_x, d_w, d_y, n, h, w, c, r, s, k, p: Conv2DParams, stream=None) -> None:
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv_fprop_f32(_ptr(d_x), _ptr(d_w), None, 0, _ptr(d_y), n, h, w, c, r, s, k,
                                               ctypes.byref(cp), 1, 1, _stream(stream)))


def launch_bprop_nhwc(d_dy, d_w, d_dx, n, h, w, c, r, s, k, p: Conv2DParams, stream=None) -> None:
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv_bprop_f32(_ptr(d_dy), _ptr(d_w), _ptr(d_dx), n, h, w, c, r, s, k,
                                               ctypes.byref(cp), 1, 1, _stream(stream)))


def launch_grad_nhwc(d_x, d_dy, d_dw, n, h, w, c, r, s, k, p: Conv2DParams, stream=None) -> None:
    cp = p.to_c()
    _lib.check(_lib.lib().b200q_conv_grad_f32(_ptr(d_x), _ptr(d_dy), _ptr(d_dw), None, 0, n, h, w, c, r, s, k,
                                              ctypes.byref(cp), 1, 1, _stream(stream)))


def launch_block_fprop_nhwc(d_x, d_w, d_y, n, h, w, c, r, s, k, p: BlockConv2DParams, d_bias=None,
                            bias_mode: BlockBiasMode = BlockBiasMode.PerBlock, stream=None) -> None:
    cp = p.conv.to_c()
    _lib.check(_lib.lib().b200q_conv_fprop_f32(_ptr(d_x), _ptr(d_w), _ptr(d_bias), int(bias_mode), _ptr(d_y), n, h, w,
                                               c, r, s, k, ctypes.byref(cp), p.block_by, p.block_bx, _stream(stream)))


def launch_block_bprop_nhwc(d_dy, d_w, d_dx, n, h, w, c, r, s, k, p: BlockConv2DParams, stream=None) -> None:
    cp = p.conv.to_c()
    _lib.check(_lib.lib().b200q_conv_bprop_f32(_ptr(d_dy), _ptr(d_w), _ptr(d_dx), n, h, w, c, r, s, k,
                                               ctypes.byref(cp), p.block_by, p.block_bx, _stream(stream)))


def launch_block_grad_nhwc(d_x, d_dy, d_dw, n, h, w, c, r, s, k, p: BlockConv2DParams, d_dbias=None,
                           bias_mode: BlockBiasMode = BlockBiasMode.PerBlock, stream=None) -> None:
    cp = p.conv.to_c()
    _lib.check(_lib.lib().b200q_conv_grad_f32(_ptr(d_x), _ptr(d_dy), _ptr(d_dw), _ptr(d_dbias), int(bias_mode), n, h,
                                              w, c, r, s, k, ctypes.byref(cp), p.block_by, p.block_bx,
                                              _stream(stream)))


def bmm_matmul(A, B, C, batch, M, N, K, trans_a=0, trans_b=0, stream=None) -> None:
    _lib.check(_lib.lib().b200q_bmm_f32(_ptr(A), _ptr(B), _ptr(C), batch, M, N, K, int(trans_a), int(trans_b),
                                        _stream(stream)))


def bmm_fprop(A, B, Y, N, W, H, C, stream=None) -> None:
    """Y[N,W,H] = A[N,W,C] @ B[N,H,C]^T (bmm.h:41-55)."""
    bmm_matmul(A, B, Y, N, W, H, C, 0, 1, stream)


def bmm_bprop_dA(dY, B, dA, N, W, H, C, stream=None) -> None:
    """dA[N,W,C] = dY[N,W,H] @ B[N,H,C]."""
    bmm_matmul(dY, B, dA, N, W, C, H, 0, 0, stream)


def bmm_bprop_dB(dY, A, dB, N, W, H, C, stream=None) -> None:
    """dB[N,H,C] = dY[N,W,H]^T @ A[N,W,C]."""
    bmm_matmul(dY, A, dB, N, H, C, W, 1, 0, stream)


def bmm_bprop(A, B, dY, dA, dB, N, W, H, C, stream=None) -> None:
    bmm_bprop_dA(dY, B, dA, N, W, H, C, stream)
    bmm_bprop_dB(dY, A, dB, N, W, H, C, stream)
