// C entry points over the reference's own CUDA implementation (test / baseline infrastructure).
//
// Compiled by oracle/Makefile together with the reference's unmodified src/cuda_kernels.cu,
// bmm.cu and src/cuda_utils.cpp into oracle/_ref/libref_gpu.so, so the reference's SIMT GPU path
// (im2col + bmm_matmul_i32 + unpack per group, cuda_kernels.cu:1336-1392) can be timed on the same
// GPU as a secondary baseline.  Nothing here is part of the product.
#include <exception>

#include "bmm.h"
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

// The reference's fp32 launchers (src/cuda_kernels.cu:767-937, bmm.cu:270-296), for timing beside
// this library's fp32 drop-ins.  op 0 = fprop (a = x, b = w, out = y), 1 = bprop (a = dy, b = w,
// out = dx), 2 = grad (a = x, b = dy, out = dw).
extern "C" int refgpu_conv_f32(int op, const float* a, const float* b, float* out, int n, int h, int w, int c, int r,
                               int s, int k, int pad, int stride, int groups) {
  try {
    Conv2DParams p;
    p.pad_h = p.pad_w = pad;
    p.stride_h = p.stride_w = stride;
    p.groups = groups;
    if (op == 0)
      launch_fprop_nhwc(a, b, out, n, h, w, c, r, s, k, p);
    else if (op == 1)
      launch_bprop_nhwc(a, b, out, n, h, w, c, r, s, k, p);
    else
      launch_grad_nhwc(a, b, out, n, h, w, c, r, s, k, p);
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

extern "C" int refgpu_bmm_f32(const float* A, const float* B, float* C, int batch, int M, int N, int K, int ta, int tb) {
  bmm_matmul(A, B, C, batch, M, N, K, ta, tb);
  return 0;
}

// The reference's int32 batched GEMM (bmm.cu:298-322), for timing beside this library's
// bmm_matmul_i32 drop-in.
extern "C" int refgpu_bmm_i32(const int32_t* A, const int32_t* B, int32_t* C, int batch, int M, int N, int K, int ta,
                              int tb) {
  bmm_matmul_i32(A, B, C, batch, M, N, K, ta, tb);
  return 0;
}
