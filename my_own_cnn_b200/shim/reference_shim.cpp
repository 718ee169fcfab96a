// The reference's own quantized-conv and int32-bmm entry points, defined over the b200q C ABI.
//
// A reference build links this file (plus libb200q.so) in place of the reference's
// src/cuda_kernels.cu quantized section and bmm.cu's bmm_matmul_i32; every declaration comes
// unchanged from the reference headers:
//   conv_quant_detail::launch_fprop_nhwc_qi32_{u8,s5}        src/conv_types.h:232-241
//   conv_quant_detail::launch_block_fprop_nhwc_qi32_{u8,s5}  src/conv_types.h:242-251
//   bmm_matmul_i32                                            bmm.h:69-74
//   launch_{,block_}{fprop,bprop,grad}_nhwc (fp32)            src/conv_types.h:287-306
//   bmm_matmul, bmm_fprop, bmm_bprop_dA/_dB, bmm_bprop (fp32)  bmm.h:36-66
// Errors become std::runtime_error, like the reference's CUDA_CHECK / infer_conv_shape.
// Launches go to the legacy default stream, as in the reference; the caller synchronizes.
#include <cstddef>
#include <stdexcept>
#include <string>

#include "b200q.h"
#include "bmm.h"
#include "conv_types.h"

namespace {

using QpU8 = nnalgebra::QuantizationParameters<nnalgebra::DataType::LinQuantU8>;
using QpS5 = nnalgebra::QuantizationParameters<nnalgebra::DataType::LinQuantS5>;

// The C ABI reads the qparams arrays with these layouts.
static_assert(sizeof(QpU8) == sizeof(b200q_qparams_u8), "LinQuantU8 qparams layout");
static_assert(offsetof(QpU8, zero_point) == offsetof(b200q_qparams_u8, zero_point), "U8 zero_point offset");
static_assert(sizeof(QpS5) == sizeof(b200q_qparams_s5), "LinQuantS5 qparams layout");
static_assert(offsetof(QpS5, zero_point) == offsetof(b200q_qparams_s5, zero_point), "S5 zero_point offset");
static_assert(static_cast<int>(nnalgebra::DataType::LinQuantU8) == B200Q_LINQUANT_U8, "DataType values");
static_assert(static_cast<int>(nnalgebra::DataType::LinQuantS5) == B200Q_LINQUANT_S5, "DataType values");

b200q_conv_params to_c(const Conv2DParams& p) {
  return b200q_conv_params{p.pad_h, p.pad_w, p.stride_h, p.stride_w, p.dilation_h, p.dilation_w, p.groups};
}

void check(int rc, const char* what) {
  if (rc != B200Q_OK) throw std::runtime_error(std::string(what) + ": " + b200q_last_error());
}

}  // namespace

namespace conv_quant_detail {

void launch_fprop_nhwc_qi32_u8(const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c, int r,
                               int s, int k, const Conv2DParams& p, const QpU8* in_qp, const QpU8* f_qp) {
  const b200q_conv_params cp = to_c(p);
  check(b200q_fprop_nhwc_qi32(B200Q_LINQUANT_U8, d_x, d_w, d_y, n, h, w, c, r, s, k, &cp, in_qp, f_qp, nullptr),
        "launch_fprop_nhwc_qi32_u8");
}

void launch_fprop_nhwc_qi32_s5(const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c, int r,
                               int s, int k, const Conv2DParams& p, const QpS5* in_qp, const QpS5* f_qp) {
  const b200q_conv_params cp = to_c(p);
  check(b200q_fprop_nhwc_qi32(B200Q_LINQUANT_S5, d_x, d_w, d_y, n, h, w, c, r, s, k, &cp, in_qp, f_qp, nullptr),
        "launch_fprop_nhwc_qi32_s5");
}

void launch_block_fprop_nhwc_qi32_u8(const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c,
                                     int r, int s, int k, const BlockConv2DParams& p, const QpU8* in_qp,
                                     const QpU8* f_qp) {
  const b200q_conv_params cp = to_c(p.conv);
  check(b200q_block_fprop_nhwc_qi32(B200Q_LINQUANT_U8, d_x, d_w, d_y, n, h, w, c, r, s, k, &cp, p.block_by,
                                    p.block_bx, in_qp, f_qp, nullptr),
        "launch_block_fprop_nhwc_qi32_u8");
}

void launch_block_fprop_nhwc_qi32_s5(const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c,
                                     int r, int s, int k, const BlockConv2DParams& p, const QpS5* in_qp,
                                     const QpS5* f_qp) {
  const b200q_conv_params cp = to_c(p.conv);
  check(b200q_block_fprop_nhwc_qi32(B200Q_LINQUANT_S5, d_x, d_w, d_y, n, h, w, c, r, s, k, &cp, p.block_by,
                                    p.block_bx, in_qp, f_qp, nullptr),
        "launch_block_fprop_nhwc_qi32_s5");
}

}  // namespace conv_quant_detail

extern "C" void bmm_matmul_i32(const int32_t* A, const int32_t* B, int32_t* C, int batch, int M, int N, int K,
                               int trans_a, int trans_b) {
  check(b200q_bmm_matmul_i32(A, B, C, batch, M, N, K, trans_a, trans_b, nullptr), "bmm_matmul_i32");
}

// ---- fp32 entry points (3 x TF32 tcgen05 GEMMs)

void launch_fprop_nhwc(const float* d_x, const float* d_w, float* d_y, int n, int h, int w, int c, int r, int s, int k,
                       const Conv2DParams& p) {
  const b200q_conv_params cp = to_c(p);
  check(b200q_conv_fprop_f32(d_x, d_w, nullptr, 0, d_y, n, h, w, c, r, s, k, &cp, 1, 1, nullptr), "launch_fprop_nhwc");
}

void launch_bprop_nhwc(const float* d_dy, const float* d_w, float* d_dx, int n, int h, int w, int c, int r, int s,
                       int k, const Conv2DParams& p) {
  const b200q_conv_params cp = to_c(p);
  check(b200q_conv_bprop_f32(d_dy, d_w, d_dx, n, h, w, c, r, s, k, &cp, 1, 1, nullptr), "launch_bprop_nhwc");
}

void launch_grad_nhwc(const float* d_x, const float* d_dy, float* d_dw, int n, int h, int w, int c, int r, int s,
                      int k, const Conv2DParams& p) {
  const b200q_conv_params cp = to_c(p);
  check(b200q_conv_grad_f32(d_x, d_dy, d_dw, nullptr, 0, n, h, w, c, r, s, k, &cp, 1, 1, nullptr),
        "launch_grad_nhwc");
}

void launch_block_fprop_nhwc(const float* d_x, const float* d_w, float* d_y, int n, int h, int w, int c, int r, int s,
                             int k, const BlockConv2DParams& p, const float* d_bias, BlockBiasMode bias_mode) {
  const b200q_conv_params cp = to_c(p.conv);
  check(b200q_conv_fprop_f32(d_x, d_w, d_bias, static_cast<int>(bias_mode), d_y, n, h, w, c, r, s, k, &cp,
                             p.block_by, p.block_bx, nullptr),
        "launch_block_fprop_nhwc");
}

void launch_block_bprop_nhwc(const float* d_dy, const float* d_w, float* d_dx, int n, int h, int w, int c, int r,
                             int s, int k, const BlockConv2DParams& p) {
  const b200q_conv_params cp = to_c(p.conv);
  check(b200q_conv_bprop_f32(d_dy, d_w, d_dx, n, h, w, c, r, s, k, &cp, p.block_by, p.block_bx, nullptr),
        "launch_block_bprop_nhwc");
}

void launch_block_grad_nhwc(const float* d_x, const float* d_dy, float* d_dw, int n, int h, int w, int c, int r,
                            int s, int k, const BlockConv2DParams& p, float* d_dbias, BlockBiasMode bias_mode) {
  const b200q_conv_params cp = to_c(p.conv);
  check(b200q_conv_grad_f32(d_x, d_dy, d_dw, d_dbias, static_cast<int>(bias_mode), n, h, w, c, r, s, k, &cp,
                            p.block_by, p.block_bx, nullptr),
        "launch_block_grad_nhwc");
}

extern "C" void bmm_matmul(const float* A, const float* B, float* C, int batch, int M, int N, int K, int trans_a,
                           int trans_b) {
  check(b200q_bmm_f32(A, B, C, batch, M, N, K, trans_a, trans_b, nullptr), "bmm_matmul");
}

// The layer API of bmm.h:41-66, in terms of bmm_matmul as the reference defines it (bmm.cu:324-361).
extern "C" void bmm_fprop(const float* A, const float* B, float* Y, int N, int W, int H, int C) {
  bmm_matmul(A, B, Y, N, W, H, C, BMM_TRANSPOSE_NONE, BMM_TRANSPOSE_YES);
}
extern "C" void bmm_bprop_dA(const float* dY, const float* B, float* dA, int N, int W, int H, int C) {
  bmm_matmul(dY, B, dA, N, W, C, H, BMM_TRANSPOSE_NONE, BMM_TRANSPOSE_NONE);
}
extern "C" void bmm_bprop_dB(const float* dY, const float* A, float* dB, int N, int W, int H, int C) {
  bmm_matmul(dY, A, dB, N, H, C, W, BMM_TRANSPOSE_YES, BMM_TRANSPOSE_NONE);
}
extern "C" void bmm_bprop(const float* A, const float* B, const float* dY, float* dA, float* dB, int N, int W, int H,
                          int C) {
  bmm_bprop_dA(dY, B, dA, N, W, H, C);
  bmm_bprop_dB(dY, A, dB, N, W, H, C);
}
