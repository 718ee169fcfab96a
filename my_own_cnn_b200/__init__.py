"""my_own_cnn_b200: B200-native (sm_100a) int8 NHWC convolution and batched GEMM, with the
reference's fp32 conv (forward and both gradients) and fp32 bmm on the same tensor-core engine.

A from-scratch implementation of the quantized conv / bmm hot path of NikitaYak02/my_own_cnn
behind the reference's own entry points.  The kernels live in ``libb200q.so`` (C ABI:
include/b200q.h); this package is the Python host side over that ABI.
"""
from .quant import (DataType, QuantizationParametersU8, QuantizationParametersS5, get_zero_point,
                    qparams_to_device)
from .conv import (Conv2DParams, BlockConv2DParams, ConvShape, BlockConvShape, Epilogue, infer_conv_shape,
                   infer_block_conv_shape, launch_fprop_nhwc_qi32, launch_block_fprop_nhwc_qi32, conv2d_s8,
                   conv2d_s8_into, conv2d_s8_add, conv2d_s8_add_into, conv2d_s8_plan, conv_out_shape)
from .pool import global_avgpool_s8, maxpool_s8
from .bmm import BMM_TRANSPOSE_NONE, BMM_TRANSPOSE_YES, bmm_matmul_i32, bmm_s8, bmm_s8_into
from .f32 import (BlockBiasMode, bmm_bprop, bmm_bprop_dA, bmm_bprop_dB, bmm_fprop, bmm_matmul, launch_block_bprop_nhwc,
                  launch_block_fprop_nhwc, launch_block_grad_nhwc, launch_bprop_nhwc, launch_fprop_nhwc,
                  launch_grad_nhwc)
from ._lib import B200QError, last_path, set_path_policy, tc_launch_count

__all__ = [
    "DataType", "QuantizationParametersU8", "QuantizationParametersS5", "get_zero_point", "qparams_to_device",
    "Conv2DParams", "BlockConv2DParams", "ConvShape", "BlockConvShape", "Epilogue", "infer_conv_shape",
    "infer_block_conv_shape", "launch_fprop_nhwc_qi32", "launch_block_fprop_nhwc_qi32", "conv2d_s8",
    "conv2d_s8_into", "conv2d_s8_add", "conv2d_s8_add_into", "conv2d_s8_plan", "maxpool_s8", "global_avgpool_s8", "conv_out_shape", "BMM_TRANSPOSE_NONE", "BMM_TRANSPOSE_YES", "bmm_matmul_i32", "bmm_s8",
    "bmm_s8_into", "B200QError", "last_path", "set_path_policy", "tc_launch_count",
    "BlockBiasMode", "launch_fprop_nhwc", "launch_bprop_nhwc", "launch_grad_nhwc", "launch_block_fprop_nhwc",
    "launch_block_bprop_nhwc", "launch_block_grad_nhwc", "bmm_matmul", "bmm_fprop", "bmm_bprop_dA", "bmm_bprop_dB",
    "bmm_bprop",
]
