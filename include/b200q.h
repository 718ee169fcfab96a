/*
 * b200q -- B200-native (sm_100a) int8 / quantized-int32 NHWC convolution and
 * batched GEMM behind a plain C ABI.
 *
 * Every entry point takes device pointers, plain sizes and a CUDA stream passed
 * as `void*` (a cudaStream_t; NULL = legacy default stream), returns an int
 * status (B200Q_OK on success) and never throws.  The message of the last
 * failure on the calling thread is returned by b200q_last_error().
 * Launches are asynchronous on `stream` unless stated otherwise.
 *
 * Drop-in mapping (reference = NikitaYak02/my_own_cnn):
 *   b200q_fprop_nhwc_qi32        replaces conv_quant_detail::launch_fprop_nhwc_qi32_{u8,s5}
 *                                (src/conv_types.h:232-241, src/cuda_kernels.cu:1336-1392,1465-1481)
 *   b200q_block_fprop_nhwc_qi32  replaces conv_quant_detail::launch_block_fprop_nhwc_qi32_{u8,s5}
 *                                (src/conv_types.h:242-251, src/cuda_kernels.cu:1394-1461,1483-1497)
 *   b200q_bmm_matmul_i32         replaces bmm_matmul_i32 (bmm.h:69-74, bmm.cu:298-322)
 *   b200q_conv_fprop_f32         replaces launch_fprop_nhwc / launch_block_fprop_nhwc
 *                                (src/conv_types.h:287-299, src/cuda_kernels.cu:767-823, 939-998)
 *   b200q_conv_bprop_f32         replaces launch_bprop_nhwc / launch_block_bprop_nhwc
 *                                (src/conv_types.h:290-302, src/cuda_kernels.cu:825-872, 1000-1057)
 *   b200q_conv_grad_f32          replaces launch_grad_nhwc / launch_block_grad_nhwc
 *                                (src/conv_types.h:293-306, src/cuda_kernels.cu:874-937, 1059-1136)
 *   b200q_bmm_f32                replaces bmm_matmul (bmm.h:36-39, bmm.cu:270-296); the layer API
 *                                bmm_fprop / bmm_bprop* (bmm.h:41-66) is defined over it by the shim
 * New entry points (int8 storage, fused requantization; no reference counterpart):
 *   b200q_conv2d_s8, b200q_bmm_s8.
 * The C++ shim my_own_cnn_b200/shim/reference_shim.cpp defines the reference's
 * own symbols on top of these, so reference callers link unchanged.
 */
#ifndef B200Q_H_
#define B200Q_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
enum b200q_status {
  B200Q_OK = 0,
  B200Q_ERR_INVALID_ARG = 1,  /* bad shape / pointer / parameter (the reference throws here) */
  B200Q_ERR_UNSUPPORTED = 2,  /* valid request this build cannot run */
  B200Q_ERR_CUDA = 3,         /* a CUDA runtime / driver call failed */
  B200Q_ERR_TIMEOUT = 4       /* a device-side wait ran out; the kernel returned early */
};

/* ---- quantized input types: same values as nnalgebra::DataType (src/nnalgebra_quantization.h:19-24) ---- */
enum b200q_qtype { B200Q_LINQUANT_U8 = 1, B200Q_LINQUANT_S5 = 2 };

/* Same layout as Conv2DParams (src/conv_types.h:21-29). */
typedef struct b200q_conv_params {
  int pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w, groups;
} b200q_conv_params;

/* Same layouts as QuantizationParameters<LinQuantU8/LinQuantS5>
 * (src/nnalgebra_quantization.h:29-41).  Only zero_point is read. */
typedef struct b200q_qparams_u8 {
  uint8_t zero_point;
  float scale;
  uint8_t symmetric; /* C++ bool */
} b200q_qparams_u8;
typedef struct b200q_qparams_s5 {
  int8_t zero_point;
  uint8_t n_bins;
  float scale;
} b200q_qparams_s5;

/* ---- output epilogue of the int8 entry points ----
 * out_kind B200Q_OUT_S32 : y[m][k] = acc + bias[k]                       (int32, wrapping; bias may be NULL)
 * out_kind B200Q_OUT_S8  : t = acc + bias[k] (int32 wrap); p = (float)t * scale[k] (fp32, RNE);
 *                          q = rint(clamp(p, clamp_lo - zp_out, clamp_hi - zp_out)) + zp_out  (half to even);
 *                          stored as int8.  ReLU = clamp_lo = zp_out; ReLU6 = clamp_hi = q6.
 * out_kind B200Q_OUT_F32 : y = (float)(acc + bias[k]) * scale[k]        (fp32, RNE)
 * For bmm, "k" is the output column n (per-column bias / scale). */
enum b200q_out_kind { B200Q_OUT_S32 = 0, B200Q_OUT_S8 = 1, B200Q_OUT_F32 = 2 };
typedef struct b200q_epilogue {
  int out_kind;
  int zp_out;
  int clamp_lo;
  int clamp_hi;
} b200q_epilogue;

/* ---- drop-in entry points ---- */

/* Quantized NHWC conv forward, int32 accumulators.
 * d_x: [n,h,w,c] float codes, d_w: [k,r,s,c/groups] float codes (cast with truncation
 * like static_cast<int32_t>), d_y: [n,ho,wo,k] int32, every element written.
 * d_in_qp: device array of n qparams (per image), d_f_qp: device pointer to one qparams,
 * of the struct type selected by qtype.
 * y = sum over valid taps of (x - zp_in[img]) * (w - zp_f), int32 wrapping.
 * Runs on tcgen05 tensor cores (raw 8-bit codes, zero points restored by per-row / per-column terms;
 * codes outside the 8-bit range fall back to a direct computation on the device), except groups of
 * (c/groups) * (k/groups) <= 16 channel pairs, which run on a direct CUDA-core kernel.  Uses the
 * stream's workspace for the 8-bit operands.
 * Replaces conv_quant_detail::launch_fprop_nhwc_qi32_{u8,s5} (src/conv_types.h:232-241). */
int b200q_fprop_nhwc_qi32(int qtype, const float* d_x, const float* d_w, int32_t* d_y, int n, int h,
                          int w, int c, int r, int s, int k, const b200q_conv_params* p,
                          const void* d_in_qp, const void* d_f_qp, void* stream);

/* Blocked variant: the filter slice is chosen by the output block
 * (by = ho / (ho_total / block_by), bx = wo / (wo_total / block_bx));
 * d_w: [k, block_by, block_bx, r, s, c/groups].
 * Replaces conv_quant_detail::launch_block_fprop_nhwc_qi32_{u8,s5} (src/conv_types.h:242-251). */
int b200q_block_fprop_nhwc_qi32(int qtype, const float* d_x, const float* d_w, int32_t* d_y, int n,
                                int h, int w, int c, int r, int s, int k,
                                const b200q_conv_params* p, int block_by, int block_bx,
                                const void* d_in_qp, const void* d_f_qp, void* stream);

/* Row-major int32 batched GEMM, C_b = op(A_b) @ op(B_b), int32 wrap-around.
 * Layouts as bmm.h:9-29.  Replaces bmm_matmul_i32 (bmm.h:69-74).
 * With 16-byte aligned A, B and C, K < 2^17 and the contiguous dimensions of A and B multiples of
 * 16, the operands are first copied to int8 in the stream's workspace and multiplied by the
 * tcgen05 GEMM (path 16); if any value lies outside [-128, 127] a device flag makes the CUDA-core
 * kernel recompute C from the int32 operands, so every input gives the same C without a host
 * round trip.  Other shapes run the CUDA-core kernel directly (path 6). */
int b200q_bmm_matmul_i32(const int32_t* A, const int32_t* B, int32_t* C, int batch, int M, int N,
                         int K, int trans_a, int trans_b, void* stream);

/* ---- fp32 drop-ins (tensor cores, 3 x TF32 split products) ----
 * All tensors fp32 in the reference's layouts: x / dx [n,h,w,c], y / dy [n,ho,wo,k],
 * w / dw [k, block_by, block_bx, r, s, c/groups] (block_by = block_bx = 1: the regular KRSC filter).
 * Each operand is split as hi + lo (hi = the value rounded to TF32's 10-bit mantissa, lo = the exact
 * remainder) and the products hi*hi + hi*lo + lo*hi are summed in fp32 by kind::tf32 tcgen05 MMAs,
 * so results agree with an fp32 loop to about 1e-6 of sum(|x||w|) per output (the tests bound the
 * difference to an exact float64 sum by 1e-5 * sum(|x||w|)).  Summation order differs from the
 * reference's loops, so results are not bit-identical to them.  Inputs are assumed finite.
 * Workspace: a per-(device, stream) grow-only buffer holding the split operands.  Groups with
 * (c/groups) * (k/groups) <= 16 (depthwise and the like) run on CUDA-core fp32 kernels instead:
 * a GEMM per group would have 1-4 rows or columns. */

/* y = conv(x, w) (+ bias of the output block).  d_bias: NULL or [k * block_by * block_bx];
 * bias_mode 0 = one bias per (k, block), 1 = one per k shared by all blocks, at index
 * k * block_by * block_bx (BlockBiasMode, src/conv_types.h:36-39, 184-188). */
int b200q_conv_fprop_f32(const float* d_x, const float* d_w, const float* d_bias, int bias_mode, float* d_y, int n,
                         int h, int w, int c, int r, int s, int k, const b200q_conv_params* p, int block_by,
                         int block_bx, void* stream);

/* dx = data gradient of the conv for dy (n, h, w, c are dx's dimensions, as in the reference). */
int b200q_conv_bprop_f32(const float* d_dy, const float* d_w, float* d_dx, int n, int h, int w, int c, int r, int s,
                         int k, const b200q_conv_params* p, int block_by, int block_bx, void* stream);

/* dw = filter gradient; d_dbias (NULL or [k * block_by * block_bx]) receives the blocked bias
 * gradient with the reference's rule (src/cpu_ref.cpp:318-371): dy summed over the block's output
 * pixels whose tap (0, 0) input lies inside the image. */
int b200q_conv_grad_f32(const float* d_x, const float* d_dy, float* d_dw, float* d_dbias, int bias_mode, int n, int h,
                        int w, int c, int r, int s, int k, const b200q_conv_params* p, int block_by, int block_bx,
                        void* stream);

/* Row-major fp32 batched GEMM, C_b = op(A_b) @ op(B_b), layouts as bmm.h:9-29. */
int b200q_bmm_f32(const float* A, const float* B, float* C, int batch, int M, int N, int K, int trans_a, int trans_b,
                  void* stream);

/* ---- new int8 entry points ---- */

/* int8 NHWC conv: d_x [n,h,w,c] int8, d_w [k,r,s,c/groups] int8, zero points 0,
 * int32 accumulation, fused epilogue (see b200q_epilogue).  d_y element type per out_kind.
 * d_bias: [k] int32 or NULL; d_scale: [k] fp32 (required for S8 / F32 outputs). */
int b200q_conv2d_s8(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias,
                    const float* d_scale, void* d_y, int n, int h, int w, int c, int r, int s,
                    int k, const b200q_conv_params* p, const b200q_epilogue* epi, void* stream);

/* b200q_conv2d_s8 with a residual add fused into the int8 epilogue (the shortcut of a ResNet /
 * MobileNetV2 block; no reference counterpart):
 *   p = fp32(acc + bias[k]) * scale[k] + fp32(res[pixel][k]) * res_scale   (IEEE steps, no fma)
 *   q = clamp(rint(p), lo - zp, hi - zp) + zp
 * d_res: int8 NHWC with the output's shape, 16-byte aligned for the tensor-core paths.  int8 outputs
 * only (B200Q_ERR_INVALID_ARG otherwise). */
int b200q_conv2d_s8_add(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias, const float* d_scale,
                        const int8_t* d_res, float res_scale, int8_t* d_y, int n, int h, int w, int c, int r,
                        int s, int k, const b200q_conv_params* p, const b200q_epilogue* epi, void* stream);

/* int8 NHWC max pool (R x S window, stride, zero-free padding: padded positions take no part).
 * Output [n, (h + 2*pad_h - r)/stride_h + 1, (w + 2*pad_w - s)/stride_w + 1, c]. */
int b200q_maxpool_s8(const int8_t* d_x, int8_t* d_y, int n, int h, int w, int c, int r, int s, int stride_h,
                     int stride_w, int pad_h, int pad_w, void* stream);

/* int8 NHWC global average pool -> [n][c]: q = clamp(rint(fp32(sum) / fp32(h*w)), -128, 127). */
int b200q_global_avgpool_s8(const int8_t* d_x, int8_t* d_y, int n, int h, int w, int c, void* stream);

/* int8 batched GEMM, layouts as bmm.h:9-29, int32 accumulation, per-column epilogue.
 * d_bias: [N] int32 or NULL; d_col_scale: [N] fp32 (required for S8 / F32 outputs). */
int b200q_bmm_s8(const int8_t* A, const int8_t* B, const int32_t* d_bias, const float* d_col_scale,
                 void* C, int batch, int M, int N, int K, int trans_a, int trans_b,
                 const b200q_epilogue* epi, void* stream);

/* Packed low-channel int8 conv that allocates nothing (no counterpart in the reference).
 * For callers that may not allocate device memory at all: for example plugins inside a runtime
 * that owns and budgets every byte of GPU memory itself, or latency-critical loops where a
 * cudaMalloc (which can synchronise the device) is not acceptable.  Same arguments, arithmetic
 * and results as b200q_conv2d_s8 on its packed path (im2col matrix + tcgen05 GEMM), for any
 * groups == 1 conv; the im2col matrix and padded weights live in one fixed 32 MiB device array
 * of this library instead of a workspace (every GPU that loads the library holds that array
 * until the process exits).  Limit: round256(N*Ho*Wo*kp) + round256(K*kp) <= 32 MiB with
 * kp = round_up(R*S*C, 32) <= 16384 (the packed path's own limit; a larger kp returns
 * B200Q_ERR_UNSUPPORTED); larger scratch requests return B200Q_ERR_INVALID_ARG with the sizes
 * in b200q_last_error().  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and keeps it for the life of the process; make that first call before
 * any stream capture, and do not reset the device (cudaDeviceReset) between calls.  All calls on a
 * device share the array: every byte the kernels read is rewritten by the same call, but calls
 * that overlap on the GPU (different streams, or host threads sharing a device) race. */
int b200q_conv2d_s8_packed_noalloc(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias,
                                   const float* d_scale, void* d_y, int n, int h, int w, int c, int r,
                                   int s, int k, const b200q_conv_params* p,
                                   const b200q_epilogue* epi, void* stream);

/* Size in bytes of the fixed scratch array behind b200q_conv2d_s8_packed_noalloc. */
size_t b200q_noalloc_scratch_bytes(void);

/* ---- host utilities ---- */

/* Kernel family (b200q_last_path code) that b200q_conv2d_s8 / b200q_conv2d_s8_add
 * (has_residual != 0) would dispatch this conv to, assuming 16-byte aligned tensor pointers and
 * the current path policy; decided on the host without launching anything (the SM count of the
 * current device, or 148 when no GPU is visible).  The same decision drives the dispatch. */
int b200q_conv2d_s8_plan(int n, int h, int w, int c, int r, int s, int k, const b200q_conv_params* p,
                         const b200q_epilogue* epi, int has_residual, int* path);

/* Output shape with the checks of infer_conv_shape (src/conv_types.h:125-146). */
int b200q_conv_out_shape(int h, int w, int c, int r, int s, int k, const b200q_conv_params* p,
                         int* ho, int* wo);

/* Message of the last failed call on this thread ("" if none). */
const char* b200q_last_error(void);

/* Synchronizes the device, then reads and clears the device-side error word that
 * kernels set when a bounded wait runs out.  Returns B200Q_OK or B200Q_ERR_TIMEOUT. */
int b200q_device_error(void);

/* Which kernel family the last conv / bmm call on this thread dispatched to:
 * 1 tcgen05 im2col conv, 2 tcgen05 tiled GEMM (for both: GEMMs of at least 2^36 MACs first prepack
 * their weights into per-stage images in the stream's workspace), 3 CUDA-core generic, 4 CUDA-core depthwise,
 * 5 CUDA-core quantized-int32 (drop-in), 6 CUDA-core int32 bmm, 7 tcgen05 GEMM over an im2col matrix
 * packed into the stream's workspace (low channel counts), 8 tcgen05 tiled GEMM on 2-SM pairs
 * (256-row tiles, one M = 256 MMA per K slice across a cluster of two CTAs), 9 tcgen05 row-tile
 * 3x3 conv (one input-window load per tile serves all nine taps), 10 tcgen05 row tiles over a
 * space-to-depth copy of a stride-2 low-channel input (network stems; the input and weights are
 * rearranged into the stream's workspace), 11 tcgen05 quantized-int32 drop-in (raw 8-bit codes and
 * zero-point correction terms), 12 CUDA-core depthwise with TMA-staged tiles, 13 tcgen05 fp32
 * (3 x TF32 split GEMM), 14 CUDA-core fp32 (groups of a few channels, e.g. depthwise), 15 tcgen05
 * pixel-grouped 1x1 GEMM (G pixels per row against block-diagonal weights built in the stream's
 * workspace, for layers with G * K <= 256 and G * C <= 256), 16 tcgen05 int32 bmm (operands copied
 * to int8, CUDA-core recompute only when a value does not fit). */
int b200q_last_path(void);

/* 0 = automatic dispatch (default); 1 = force the CUDA-core kernels (cross-checks). */
void b200q_set_path_policy(int policy);

/* Number of tcgen05 GEMM launches, and of the weight-prepack launches that feed them, issued since
   load (for launch accounting). */
long long b200q_tc_launch_count(void);

/* ---- seeded synthetic data (counter-based splitmix64; the CPU oracle regenerates any slice) ---- */
int b200q_fill_s8_uniform(int8_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id, int lo,
                          int hi, void* stream);
int b200q_fill_i32_uniform(int32_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id,
                           int32_t lo, int32_t hi, void* stream);
/* d_table: 65536 int8 codes in device memory (quantiles of the wanted distribution). */
int b200q_fill_s8_table(int8_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id,
                        const int8_t* d_table, void* stream);

/* Failure-path self test: one CTA waits on an mbarrier that nothing completes, with a
 * limit of `cycles` SM clocks, then records a timeout and returns.  Synchronous.
 * Returns B200Q_ERR_TIMEOUT when the bounded wait behaved (the expected result). */
int b200q_selftest_wait_timeout(long long cycles);

#ifdef __cplusplus
}
#endif

#endif /* B200Q_H_ */
