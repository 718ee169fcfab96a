// C entry points over the reference's own CUDA implementation (test / baseline infrastructure).
//
// Compiled by oracle/Makefile together with the reference's unmodified src/cuda_kernels.cu,
// bmm.cu and src/cuda_utils.cpp into oracle/_ref/libref_gpu.so, so the reference's SIMT GPU path
// (im2col + bmm_matmul_i32 + unpack per group, cuda_kernels.cu:1336-1392) can be timed on the same
// GPU as a secondary baseline.  Nothing here is part of the product.
#include <exception>

#include "conv_types.h"

extern "C" int refgpu_fprop_qi32_s5(const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c,
                                    int r, int s, int k, int pad, int stride, const void* d_in_qp,
                                    const void* d_f_qp) {
  using QP = nnalgebra::QuantizationParameters<nnalgebra::DataType::LinQuantS5>;
  try {
    Conv2DParams p;
    p.pad_h = p.pad_w = pad;
    p.stride_h = p.stride_w = stride;
    launch_fprop_nhwc_qi32<nnalgebra::DataType::LinQuantS5>(d_x, d_w, d_y, n, h, w, c, r, s, k, p,
                                                           static_cast<const QP*>(d_in_qp),
                                                           static_cast<const QP*>(d_f_qp));
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}
