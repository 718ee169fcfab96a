// b200q: host side of the C ABI declared in include/b200q.h.
//
// Validation follows the reference's own checks (infer_conv_shape / infer_block_conv_shape,
// src/conv_types.h:125-169) but returns status codes instead of throwing.  Dispatch:
//   conv2d_s8 : tcgen05 implicit GEMM (im2col TMA, or plain tiled TMA for 1x1/s1/p0) when
//               groups == 1, C % 16 == 0 and the tensors are 16-byte aligned (channels past C in
//               the last K block are zero-filled by TMA in both operands);
//               depthwise CUDA-core kernel for groups == C == K, C % 16 == 0;
//               low channel counts (C % 16 != 0, e.g. the C = 3 stems): im2col pack into a
//               per-stream workspace + the same tcgen05 GEMM;
//               CUDA-core direct kernel otherwise.
//   bmm_s8    : tcgen05 tiled GEMM (K-major or MN-major operands) when the TMA stride rules hold,
//               CUDA-core tiled GEMM otherwise.
//   *_qi32 drop-ins and bmm_matmul_i32: float codes / int32 values copied to 8-bit operands for the
//               tcgen05 GEMM, with a device flag that reruns exact CUDA-core kernels when a value
//               does not fit the 8-bit operand type.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/b200q.h"
#include "common.cuh"
#include "simt.cuh"
#include "tc_gemm.cuh"
#include "qi32_tc.cuh"
#include "dw_tma.cuh"
#include "f32_tc.cuh"

namespace b200q {
namespace {

thread_local char g_errmsg[512] = "";
thread_local int g_last_path = 0;
std::atomic<int> g_policy{0};
std::atomic<long long> g_tc_launches{0};
std::atomic<uint32_t> g_flag_gen{0};

// Nonzero number of a drop-in call; its out-of-range flag is set to this value, so a flag left by an
// earlier call (or uninitialised workspace) does not need a clearing copy before each call.
int next_flag_gen() {
  uint32_t v;
  do v = (g_flag_gen.fetch_add(1) + 1) & 0x7fffffffu; while (v == 0);
  return static_cast<int>(v);
}

__device__ int g_dev_err;

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_errmsg, sizeof(g_errmsg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B200Q_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// --------------------------------------------------------------- per-device state
struct DeviceState {
  bool init = false;
  int sms = 0;
  int* err = nullptr;  // device address of g_dev_err
};
DeviceState g_dev[64];
std::mutex g_dev_mu;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
typedef CUresult (*EncodeIm2colFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const int*, const int*, cuuint32_t, cuuint32_t,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode_tiled = nullptr;
EncodeIm2colFn g_encode_im2col = nullptr;

long long wait_limit() {
  static long long v = [] {
    const char* s = getenv("B200Q_WAIT_LIMIT_CYCLES");
    long long x = s ? atoll(s) : 0;
    return x > 0 ? x : (1ll << 31);  // ~1 s of SM clocks
  }();
  return v;
}

int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200Q_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& st = g_dev[dev];
  if (!st.init) {
    e = cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.err), g_dev_err);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_dev_err)");
    e = cudaFuncSetAttribute(tc_gemm_s8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc_gemm_s8_kernel)");
    e = cudaFuncSetAttribute(tc_gemm_s8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(tc_gemm_s8_pair_kernel)");
    {
      const void* dw_kernels[6] = {(const void*)dw_tma_s8_kernel<1, 0>, (const void*)dw_tma_s8_kernel<1, 1>,
                                   (const void*)dw_tma_s8_kernel<1, 2>, (const void*)dw_tma_s8_kernel<2, 0>,
                                   (const void*)dw_tma_s8_kernel<2, 1>, (const void*)dw_tma_s8_kernel<2, 2>};
      for (const void* k : dw_kernels) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(dw_tma_s8_kernel)");
      }
    }
    if (!g_encode_tiled) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
      g_encode_tiled = reinterpret_cast<EncodeTiledFn>(fn);
      fn = nullptr;
      e = cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeIm2col unavailable");
      g_encode_im2col = reinterpret_cast<EncodeIm2colFn>(fn);
    }
    st.init = true;
  }
  *out = &st;
  return B200Q_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int grid_for(size_t total, int threads, int sms) {
  size_t blocks = (total + threads - 1) / threads;
  size_t cap = static_cast<size_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return B200Q_OK;
}

int make_epilogue(const b200q_epilogue* epi, const int32_t* bias, const float* scale, Epilogue* out) {
  if (!epi) return fail(B200Q_ERR_INVALID_ARG, "epilogue descriptor is null");
  if (epi->out_kind < 0 || epi->out_kind > 2) return fail(B200Q_ERR_INVALID_ARG, "bad out_kind %d", epi->out_kind);
  if (epi->out_kind != B200Q_OUT_S32 && !scale)
    return fail(B200Q_ERR_INVALID_ARG, "int8 / fp32 outputs need per-channel scales");
  if (epi->out_kind == B200Q_OUT_S8) {
    if (epi->clamp_lo > epi->clamp_hi || epi->clamp_lo < -128 || epi->clamp_hi > 127)
      return fail(B200Q_ERR_INVALID_ARG, "int8 clamp bounds [%d,%d] invalid", epi->clamp_lo, epi->clamp_hi);
    if (epi->zp_out < -128 || epi->zp_out > 127) return fail(B200Q_ERR_INVALID_ARG, "zp_out out of int8 range");
  }
  out->out_kind = epi->out_kind;
  out->zp = epi->zp_out;
  out->lo = epi->clamp_lo;
  out->hi = epi->clamp_hi;
  out->bias = bias;
  out->scale = scale;
  out->res = nullptr;
  out->res_scale = 0.0f;
  out->rowterm = nullptr;
  out->rowzx = nullptr;
  return B200Q_OK;
}

size_t out_elem_size(int kind) { return kind == B200Q_OUT_S8 ? 1 : 4; }

// ------------------------------------------------------------------ TMA maps
int encode_tiled_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint32_t b0,
                    uint32_t b1, int swizzle_bytes, uint32_t b2 = 1) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0, d0 * d1};  // bytes (uint8 elements)
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                              es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) dims %llu,%llu,%llu box %u,%u", (int)r,
                (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, b0, b1);
  return B200Q_OK;
}

// Output map for 4-byte results: dims {N, M, batch} (int32 elements), box {32, 32, 1}, 128B swizzle.
int encode_out_4b(CUtensorMap* map, void* base, uint64_t n, uint64_t m, uint64_t batch) {
  cuuint64_t dims[3] = {n, m, batch};
  cuuint64_t strides[2] = {n * 4, n * m * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, base, dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return B200Q_OK;
}

// int8 output [batch][M][N] as a 3-D map with 32 x 32 boxes and the 32-byte swizzle of the
// epilogue's staging buffers.
int encode_out_1b(CUtensorMap* map, void* base, uint64_t n, uint64_t m, uint64_t batch, bool wide = false) {
  cuuint64_t dims[3] = {n, m, batch};
  cuuint64_t strides[2] = {n, n * m};
  cuuint32_t box[3] = {wide ? 128u : 32u, 32, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, base, dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (int8 output) failed (%d)", (int)r);
  return B200Q_OK;
}

// Row-tile window map over x [N][H][W][C]: dims {16 B, W, H, C/16, N}, box {16, P, T + 3, C/16, 1},
// no swizzle: one box lands as [C/16][T+3 rows][P columns][16 B].
// Row-tile window map of an NHWC int8 tensor: dims {16 B, w, h, c / 16, n}, box of `rows` rows x
// P pixels x all channel planes, no swizzle (shared layout [c / 16][row * P + pixel][16 B]).
int encode_rowtile(CUtensorMap* map, const int8_t* x, int n, int h, int w, int c, int P, int rows) {
  cuuint64_t dims[5] = {16, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)(c / 16), (cuuint64_t)n};
  cuuint64_t strides[4] = {(cuuint64_t)c, (cuuint64_t)c * w, 16, (cuuint64_t)c * w * h};
  cuuint32_t box[5] = {16, (cuuint32_t)P, (cuuint32_t)rows, (cuuint32_t)(c / 16), 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<int8_t*>(x), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (row-tile window) failed (%d)", (int)r);
  return B200Q_OK;
}

// Row-tile window map of a 16-channel NHWC int8 tensor read in 8-byte elements: dims
// {2 * w, h, n}, box {2 * P, rows, 1}, so each box row is P whole pixels (16 * P contiguous
// bytes) and a window takes `rows` TMA rows instead of rows * P 16-byte ones.  Shared layout
// [row * P + pixel][16 B], the same as encode_rowtile's for one channel plane.
int encode_rowtile_wide(CUtensorMap* map, const int8_t* x, int n, int h, int w, int P, int rows) {
  cuuint64_t dims[3] = {(cuuint64_t)(2 * w), (cuuint64_t)h, (cuuint64_t)n};
  cuuint64_t strides[2] = {(cuuint64_t)w * 16, (cuuint64_t)w * h * 16};
  cuuint32_t box[3] = {(cuuint32_t)(2 * P), (cuuint32_t)rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<int8_t*>(x), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (wide row-tile window) failed (%d)", (int)r);
  return B200Q_OK;
}

int encode_im2col(CUtensorMap* map, const int8_t* x, const ConvGeom& g, int bk) {
  cuuint64_t dims[4] = {(cuuint64_t)g.c, (cuuint64_t)g.w, (cuuint64_t)g.h, (cuuint64_t)g.n};
  cuuint64_t strides[3] = {(cuuint64_t)g.c, (cuuint64_t)g.c * g.w, (cuuint64_t)g.c * g.w * g.h};
  int lower[2] = {-g.pad_w, -g.pad_h};
  int upper[2] = {g.pad_w - (g.s - 1) * g.dil_w, g.pad_h - (g.r - 1) * g.dil_h};
  cuuint32_t es[4] = {1, (cuuint32_t)g.stride_w, (cuuint32_t)g.stride_h, 1};
  CUtensorMapSwizzle sw = bk == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : bk == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                     : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = g_encode_im2col(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(x), dims, strides, lower,
                               upper, (cuuint32_t)bk, (cuuint32_t)kTcBM, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d)", (int)r);
  return B200Q_OK;
}

// ------------------------------------------------------------- tcgen05 launch
constexpr int kSmemLimit = 227 * 1024;
constexpr int kSmemReserve = 1024 + 512;  // alignment slack + barriers / TMEM slot

int pick_bn(int n, int mn_major_b) {
  if (mn_major_b) return n <= 128 ? 128 : 256;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

// int8 TMA-store epilogue switch (env B200Q_S8_TMA_STORE=0 turns it off, for A/B timing).
// Wide int8 TMA stores (TcArgs::wide_store): env B200Q_S8_WIDE = 0 off, 1 reductions of at most
// B200Q_S8_WIDE_MAX_RED bytes (default 256), 2 every eligible GEMM.
const int g_s8_wide = [] {
  const char* v = getenv("B200Q_S8_WIDE");
  return v ? atoi(v) : 1;
}();

const int g_s8_wide_max_red = [] {
  const char* v = getenv("B200Q_S8_WIDE_MAX_RED");
  return v ? atoi(v) : 256;
}();

const bool g_s8_tma_store = [] {
  const char* v = getenv("B200Q_S8_TMA_STORE");
  return !(v && v[0] == '0');
}();

// Resident-B switch (env B200Q_B_RESIDENT=0 turns it off, for A/B timing).
const bool g_b_resident = [] {
  const char* v = getenv("B200Q_B_RESIDENT");
  return !(v && v[0] == '0');
}();

// 2-SM tiles switch (env B200Q_PAIR=0 turns them off, for A/B timing).
const bool g_pair = [] {
  const char* v = getenv("B200Q_PAIR");
  return !(v && v[0] == '0');
}();

// TMA-staged depthwise switch (env B200Q_DW_TMA=0 keeps the register-window kernel, for A/B timing).
const bool g_dw_tma = [] {
  const char* v = getenv("B200Q_DW_TMA");
  return !(v && v[0] == '0');
}();

// Depthwise pixels-per-thread switch (env B200Q_DW_PX=0 keeps one pixel per thread, for A/B).
const bool g_dw_px = [] {
  const char* v = getenv("B200Q_DW_PX");
  return !(v && v[0] == '0');
}();

// Word-wise pack switch (env B200Q_PACK_WORDS=0 keeps the byte-wise pack, for A/B timing).
const bool g_pack_words = [] {
  const char* v = getenv("B200Q_PACK_WORDS");
  return !(v && v[0] == '0');
}();

// Row-tile switch (env B200Q_ROWTILE=0 keeps 3x3 convs on the im2col mode, for A/B timing).
const bool g_rowtile = [] {
  const char* v = getenv("B200Q_ROWTILE");
  return !(v && v[0] == '0');
}();

// Shortest reduction of an int8-output GEMM that takes 2-SM tiles (env B200Q_PAIR_MIN_K, for A/B).
const int g_pair_min_k = [] {
  const char* v = getenv("B200Q_PAIR_MIN_K");
  return v ? atoi(v) : 2048;
}();

// Row groups per space-to-depth row tile, at most (env B200Q_RT_GROUPS, for A/B timing; 1 = one
// group; the tensor-memory cap 256 / BN applies: 4 groups of 64 columns, 8 of 32).
const int g_rt_groups = [] {
  const char* v = getenv("B200Q_RT_GROUPS");
  const int n = v ? atoi(v) : 8;
  return n < 1 ? 1 : (n > 8 ? 8 : n);
}();

// Space-to-depth stem switch (env B200Q_S2D=0 keeps low-channel stride-2 convs on the packed
// path, for A/B timing).
const bool g_s2d = [] {
  const char* v = getenv("B200Q_S2D");
  return !(v && v[0] == '0');
}();

const int g_nacc_max = [] {
  const char* v = getenv("B200Q_NACC_MAX");
  const int n = v ? atoi(v) : 8;
  return n >= 8 ? 8 : n >= 4 ? 4 : 2;
}();

// 2-SM tiles for large tiled GEMMs with more than one 256-column N tile: K-major operands, no
// channel-padding weight map, enough 256-row tiles to give every SM pair work.  Measured faster
// for reductions of 2048 and more or 4-byte outputs (config 4b +16 %); equal or slower for int8
// outputs of shorter reductions, where both CTAs' epilogues gate every accumulator buffer.  The
// caller encodes the B map with BN / 2 rows per box when this holds.
// Prepacked conv weights for long reductions (env B200Q_B_PREPACK=0: off; B200Q_PREPACK_MIN_KB:
// the shortest reduction, in 128-byte K blocks, that takes it).
const bool g_b_prepack = [] {
  const char* v = getenv("B200Q_B_PREPACK");
  return !(v && v[0] == '0');
}();
const int g_prepack_min_kb = [] {
  const char* v = getenv("B200Q_PREPACK_MIN_KB");
  return v ? atoi(v) : 8;
}();

// 2-SM tiles for batched GEMMs (bmm), either B layout (env B200Q_PAIR_BMM=0: off).
const bool g_pair_bmm = [] {
  const char* v = getenv("B200Q_PAIR_BMM");
  return !(v && v[0] == '0');
}();

bool want_pair(int sms, const TcArgs& a) {
  if (!g_pair || a.mode != 0 || a.a_major != 0 || a.conv_b || a.BN != 256) return false;
  if (a.b_major != 0 && !(g_pair_bmm && a.b_batched && a.BK == 128)) return false;
  if (a.b_batched ? !g_pair_bmm : (a.num_kb * a.BK < g_pair_min_k && a.epi.out_kind == kOutS8)) return false;
  const long long n_tiles = (a.N + a.BN - 1) / a.BN;
  const long long pair_tiles = static_cast<long long>(a.batch) * ((a.M + 2 * kTcBM - 1) / (2 * kTcBM)) * n_tiles;
  return n_tiles >= 2 && pair_tiles >= sms;
}

int launch_tc(const DeviceState& st, const CUtensorMap& ma, const CUtensorMap& mb, TcArgs a, cudaStream_t stream,
              const CUtensorMap* ma2 = nullptr) {
  // 4-byte outputs go through shared memory and TMA stores when the row pitch allows a tensor map.
  CUtensorMap mc = ma;  // unused placeholder when tma_store == 0
  a.tma_store = 0;
  if (a.mode != 2 && a.epi.out_kind != kOutS8 && a.ldc == a.N && a.N % 4 == 0 && aligned16(a.out)) {
    const uint64_t rows = a.batch_stride ? static_cast<uint64_t>(a.M) : static_cast<uint64_t>(a.M);
    int rc = encode_out_4b(&mc, a.out, static_cast<uint64_t>(a.N), rows, static_cast<uint64_t>(a.batch));
    if (rc) return rc;
    a.tma_store = 1;
  }
  a.n_tiles = (a.N + a.BN - 1) / a.BN;
  // Resident B for a single N tile whose K blocks fit in 64 KiB (narrow layers, 3x3 convs with
  // few output channels): the weights are loaded once per CTA instead of once per 128-row tile.
  const long long b_all = static_cast<long long>(a.num_kb) * a.BN * a.BK;
  a.b_res = a.mode == 2 || (!a.pair && !a.tf32 && g_b_resident && a.n_tiles == 1 && !a.b_batched && a.b_major == 0 &&
                            b_all <= 64 * 1024);
  const int b_rows = a.pair ? a.BN / 2 : a.BN;  // B rows per stage held by this CTA
  const int stage_bytes = (a.mode == 2 ? a.rt_stage : kTcBM * a.BK) + (a.b_res ? 0 : b_rows * a.BK);
  // Stage per-column bias / scale in shared memory when they fit (4096 columns = 32 KiB).
  a.stage_cols = (a.epi.out_kind != kOutS32 || a.epi.bias) && a.N <= 4096 ? (a.N + 31) / 32 * 32 : 0;
  a.default_clamp = a.epi.out_kind == kOutS8 && a.epi.zp == 0 && a.epi.lo == -128 && a.epi.hi == 127;
  a.hi_f = static_cast<float>(a.epi.hi);
  a.vec8_ok = a.epi.out_kind == kOutS8 && a.stage_cols > 0 && a.N % 8 == 0 && a.ldc % 8 == 0 &&
              reinterpret_cast<uintptr_t>(a.out) % 8 == 0 &&
              (!a.epi.res || reinterpret_cast<uintptr_t>(a.epi.res) % 8 == 0);
  // int8 outputs: TMA stores when the row pitch allows a map and every 32-column chunk can read
  // its bias / scale (staged columns are zero-padded to a multiple of 32).  GEMMs with a reduction
  // shorter than 128 are store-bound: they take the 128-byte-wide boxes (256-column tiles) or keep
  // direct stores (32-byte boxes measured no faster there); longer reductions keep the 32-byte
  // boxes, whose smaller staging leaves more ring stages.
  const bool short_red = a.num_kb * a.BK < 128;
  a.wide_store = 0;
  if (a.mode != 2 && a.epi.out_kind == kOutS8 && g_s8_tma_store && !a.pair && kTcEpiPerQuarter == 2 &&
      (g_s8_wide == 2 || (g_s8_wide == 1 && a.num_kb * a.BK <= g_s8_wide_max_red)) && a.BN == 256 &&
      a.N % 16 == 0 && a.ldc == a.N &&
      aligned16(a.out) && a.stage_cols > 0 && a.vec_ok) {
    const uint64_t rows = static_cast<uint64_t>(a.M);
    int rc = encode_out_1b(&mc, a.out, static_cast<uint64_t>(a.N), rows, static_cast<uint64_t>(a.batch), true);
    if (rc) return rc;
    a.tma_store = 1;
    a.wide_store = 1;
  } else if (a.mode != 2 && a.epi.out_kind == kOutS8 && g_s8_tma_store && !short_red && a.ldc == a.N &&
             a.N % 16 == 0 && aligned16(a.out) && (a.stage_cols > 0 || a.N % 32 == 0) && a.vec_ok) {
    const uint64_t rows = static_cast<uint64_t>(a.M);
    int rc = encode_out_1b(&mc, a.out, static_cast<uint64_t>(a.N), rows, static_cast<uint64_t>(a.batch));
    if (rc) return rc;
    a.tma_store = 1;
  }
  const int stage_out =
      a.epi.out_kind == kOutS8 ? (a.wide_store ? kEpiStageBytesS8W : kEpiStageBytesS8) : kEpiStageBytes;
  const int epi_bytes = a.stage_cols * 8 + (a.tma_store ? 1024 + kTcEpiWarps * 2 * stage_out : 0);
  const int b_res_bytes = a.b_res ? static_cast<int>(b_all) : 0;
  int stages = (kSmemLimit - kSmemReserve - epi_bytes - b_res_bytes) / stage_bytes;
  if (stages > 8) stages = 8;
  if (stages < 2) return fail(B200Q_ERR_UNSUPPORTED, "tile does not fit shared memory");
  a.stages = stages;
  const int tile_m = a.pair ? 2 * kTcBM : kTcBM;
  if (a.rt_G < 1) a.rt_G = 1;
  a.m_tiles = a.mode == 2 ? a.n_img * ((a.Ho + a.rt_T * a.rt_G - 1) / (a.rt_T * a.rt_G)) : (a.M + tile_m - 1) / tile_m;
  const long long total = static_cast<long long>(a.batch) * a.m_tiles * a.n_tiles;
  if (total > 0x7FFFFFFFll) return fail(B200Q_ERR_UNSUPPORTED, "too many tiles");
  a.total_tiles = static_cast<int>(total);
  // As many accumulator buffers as the 512 TMEM columns hold: short reductions finish a tile
  // every few hundred cycles, and the MMA warp must not wait for the epilogue's turnaround.
  a.acc_cols = a.BN * a.rt_G;
  a.nacc = g_nacc_max < 512 / a.acc_cols ? g_nacc_max : 512 / a.acc_cols;
  if (a.nacc < 2) return fail(B200Q_ERR_UNSUPPORTED, "accumulator does not fit tensor memory twice");
  // tcgen05.alloc takes a power of two of at least 32 columns (row groups of 3, 5, 6 or 7 give
  // buffers of 192, 320, ... columns): allocate the next power of two, at most the 512 columns.
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(a.nacc * a.acc_cols)) cols <<= 1;
  a.tmem_cols = cols;
  const uint32_t sgn = a.ab_unsigned ? 0u : 1u;       // kind::i8 operand type: 0 = u8, 1 = s8
  const uint32_t dfmt = a.tf32 ? 1u : 2u;               // D = f32 (kind::tf32) or s32 (kind::i8)
  const uint32_t abfmt = a.tf32 ? 2u : sgn;             // kind::tf32 operand format: 2 = TF32
  a.idesc = (dfmt << 4)
            | (abfmt << 7) | (abfmt << 10)              // A, B type
            | (static_cast<uint32_t>(a.a_major) << 15)  // A major
            | (static_cast<uint32_t>(a.b_major) << 16)  // B major
            | (static_cast<uint32_t>(a.BN >> 3) << 17)  // N
            | (static_cast<uint32_t>(tile_m >> 4) << 24);  // M (256 for the pair MMA)
  a.wait_limit = wait_limit();
  a.err = st.err;
  int grid = a.total_tiles < st.sms ? a.total_tiles : st.sms;
  if (a.pair) grid = 2 * (a.total_tiles < st.sms / 2 ? a.total_tiles : st.sms / 2);
  size_t smem = static_cast<size_t>(stages) * stage_bytes + b_res_bytes + kSmemReserve + epi_bytes;
  // One CTA per SM: the CTA allocates all 512 TMEM columns, so a second resident CTA of this
  // grid would only wait for them.  Asking for more than half the shared memory rules it out.
  if (smem < static_cast<size_t>(kSmemLimit / 2 + 1024)) smem = kSmemLimit / 2 + 1024;
  if (a.pair) {
    tc_gemm_s8_pair_kernel<<<grid, kTcThreads, smem, stream>>>(ma, mb, mc, a);
    g_tc_launches.fetch_add(1, std::memory_order_relaxed);
    return check_launch("tc_gemm_s8_pair_kernel launch");
  }
  tc_gemm_s8_kernel<<<grid, kTcThreads, smem, stream>>>(ma, mb, mc, a, ma2 ? *ma2 : ma);
  g_tc_launches.fetch_add(1, std::memory_order_relaxed);
  return check_launch("tc_gemm_s8_kernel launch");
}

int conv_geom(int n, int h, int w, int c, int r, int s, int k, const b200q_conv_params* p, int by, int bx,
              ConvGeom* g) {
  if (!p) return fail(B200Q_ERR_INVALID_ARG, "conv params pointer is null");
  if (n <= 0 || h <= 0 || w <= 0 || c <= 0 || r <= 0 || s <= 0 || k <= 0)
    return fail(B200Q_ERR_INVALID_ARG, "tensor dimensions must be > 0");
  if (p->dilation_h <= 0 || p->dilation_w <= 0) return fail(B200Q_ERR_INVALID_ARG, "dilation must be > 0");
  if (p->pad_h < 0 || p->pad_w < 0) return fail(B200Q_ERR_INVALID_ARG, "padding must be >= 0");
  int ho = 0, wo = 0;
  int rc = b200q_conv_out_shape(h, w, c, r, s, k, p, &ho, &wo);
  if (rc) return rc;
  if (by <= 0 || bx <= 0) return fail(B200Q_ERR_INVALID_ARG, "block_by and block_bx must be > 0");
  if (ho % by || wo % bx) return fail(B200Q_ERR_INVALID_ARG, "blocked convolution requires Ho/Wo divisible by block grid");
  g->n = n; g->h = h; g->w = w; g->c = c; g->r = r; g->s = s; g->k = k; g->ho = ho; g->wo = wo;
  g->pad_h = p->pad_h; g->pad_w = p->pad_w; g->stride_h = p->stride_h; g->stride_w = p->stride_w;
  g->dil_h = p->dilation_h; g->dil_w = p->dilation_w; g->groups = p->groups;
  g->cg = c / p->groups; g->kg = k / p->groups;
  g->by = by; g->bx = bx; g->bho = ho / by; g->bwo = wo / bx;
  const long long total = static_cast<long long>(n) * ho * wo * k;
  if (total > (1ll << 46)) return fail(B200Q_ERR_UNSUPPORTED, "output too large");
  return B200Q_OK;
}

int get_workspace(size_t bytes, cudaStream_t stream, void** out);
size_t round256(size_t v);

// Tensor-core route of the drop-in (see qi32_tc.cuh): pack 8-bit rows and filter rows with their
// zero-point terms, one batched tcgen05 GEMM over (output block x group), then the correction /
// scatter pass.  Returns B200Q_ERR_UNSUPPORTED (nothing launched) for shapes it does not take.
int qi32_tensor_core(const DeviceState& st, int qtype, const float* x, const float* w, int32_t* y, const ConvGeom& g,
                     const void* in_qp, const void* f_qp, cudaStream_t stream) {
  Qi32Pack q{};
  q.T = g.r * g.s * g.cg;
  q.kp = (q.T + 31) / 32 * 32;
  q.gcount = g.by * g.bx * g.groups;
  const long long mb = static_cast<long long>(g.n) * g.bho * g.bwo;
  q.qp_stride = qtype == B200Q_LINQUANT_U8 ? (int)sizeof(b200q_qparams_u8) : (int)sizeof(b200q_qparams_s5);
  q.qp_signed = qtype == B200Q_LINQUANT_S5;
  if (q.kp > 16384 || mb >= (1ll << 31) || static_cast<long long>(q.gcount) * mb >= (1ll << 40))
    return B200Q_ERR_UNSUPPORTED;
  q.mb = static_cast<int>(mb);
  const long long arows = static_cast<long long>(q.gcount) * mb;
  const long long brows = static_cast<long long>(q.gcount) * g.kg;
  const bool in_place = q.gcount == 1;  // the GEMM writes y directly; the fixup corrects in place
  const size_t a_bytes = round256(static_cast<size_t>(arows) * q.kp);
  const size_t b_bytes = round256(static_cast<size_t>(brows) * q.kp);
  const size_t rt_bytes = round256(static_cast<size_t>(arows) * 4) * 2;  // row terms, then row zero points
  const size_t cs_bytes = round256(static_cast<size_t>(brows) * 4);
  const size_t c_bytes = in_place ? 0 : round256(static_cast<size_t>(arows) * g.kg * 4);
  void* ws = nullptr;
  int rc = get_workspace(a_bytes + b_bytes + rt_bytes + cs_bytes + c_bytes + 256, stream, &ws);
  if (rc) return rc;
  uint8_t* base = static_cast<uint8_t*>(ws);
  uint32_t* a_buf = reinterpret_cast<uint32_t*>(base);
  uint32_t* b_buf = reinterpret_cast<uint32_t*>(base + a_bytes);
  int32_t* rowterm = reinterpret_cast<int32_t*>(base + a_bytes + b_bytes);
  int32_t* rowzx = reinterpret_cast<int32_t*>(base + a_bytes + b_bytes + rt_bytes / 2);
  int32_t* colsum = reinterpret_cast<int32_t*>(base + a_bytes + b_bytes + rt_bytes);
  int32_t* cbuf = in_place ? y : reinterpret_cast<int32_t*>(base + a_bytes + b_bytes + rt_bytes + cs_bytes);
  int* flag = reinterpret_cast<int*>(base + a_bytes + b_bytes + rt_bytes + cs_bytes + c_bytes);
  q.gen = next_flag_gen();  // the flag is not cleared: the kernels compare it with this call's number
  const uint8_t* iq = static_cast<const uint8_t*>(in_qp);
  const uint8_t* fq = static_cast<const uint8_t*>(f_qp);
  const int row_blocks = grid_for(static_cast<size_t>(arows) * 32, 256, st.sms);
  const int filter_blocks = grid_for(static_cast<size_t>(brows) * 32, 256, st.sms);
  if (a_bytes + b_bytes <= (8u << 20)) {
    // small problems are launch-latency-bound: both packs in one launch (config 1: 34.8 -> 28.7 us
    // per call); large ones measured 3-7 % faster as two launches
    qi32_pack_kernel<<<row_blocks + filter_blocks, 256, 0, stream>>>(x, a_buf, rowterm, rowzx, w, b_buf, colsum, g,
                                                                     q, iq, fq, flag, row_blocks);
    rc = check_launch("qi32_pack_kernel launch");
    if (rc) return rc;
  } else {
    qi32_pack_rows_kernel<<<row_blocks, 256, 0, stream>>>(x, a_buf, rowterm, rowzx, g, q, iq, fq, flag);
    rc = check_launch("qi32_pack_rows_kernel launch");
    if (rc) return rc;
    qi32_pack_filter_kernel<<<filter_blocks, 256, 0, stream>>>(w, b_buf, colsum, g, q, flag);
    rc = check_launch("qi32_pack_filter_kernel launch");
    if (rc) return rc;
  }
  TcArgs a{};
  a.mode = 0;
  a.BK = q.kp % 128 == 0 ? 128 : (q.kp % 64 == 0 ? 64 : 32);
  a.BN = pick_bn(g.kg, 0);
  a.M = q.mb;
  a.N = g.kg;
  a.batch = q.gcount;
  a.b_batched = q.gcount > 1;
  a.num_kb = q.kp / a.BK;
  a.epi = Epilogue{kOutS32, 0, 0, 0, nullptr, nullptr, nullptr, 0.0f};
  if (in_place) {  // one block, one group: the correction goes into the GEMM epilogue
    a.epi.bias = colsum;
    a.epi.rowterm = rowterm;
    a.epi.rowzx = rowzx;
  }
  a.out = cbuf;
  a.ldc = g.kg;
  a.batch_stride = static_cast<long long>(q.mb) * g.kg;
  a.vec_ok = g.kg % 16 == 0 && aligned16(cbuf);
  a.ab_unsigned = qtype == B200Q_LINQUANT_U8;
  CUtensorMap ma, mb_map;
  rc = encode_tiled_3d(&ma, a_buf, static_cast<uint64_t>(q.kp), static_cast<uint64_t>(q.mb),
                       static_cast<uint64_t>(q.gcount), a.BK, kTcBM, a.BK);
  if (rc) return rc;
  a.pair = want_pair(st.sms, a);
  rc = encode_tiled_3d(&mb_map, b_buf, static_cast<uint64_t>(q.kp), static_cast<uint64_t>(g.kg),
                       static_cast<uint64_t>(q.gcount), a.BK, a.pair ? a.BN / 2 : a.BN, a.BK);
  if (rc) return rc;
  rc = launch_tc(st, ma, mb_map, a, stream);
  if (rc) return rc;
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  const bool v4 = g.kg % 4 == 0 && aligned16(y) && aligned16(cbuf);
  const int fused = in_place ? 1 : 0;
  // fused: the launch only serves the out-of-range fallback, so one block per SM (grid-stride loop)
  // keeps it cheap while the flag is clear
  const int gv4 = fused ? std::min(grid_for(total / 4, 256, st.sms), st.sms) : grid_for(total / 4, 256, st.sms);
  const int gv1 = fused ? std::min(grid_for(total, 256, st.sms), st.sms) : grid_for(total, 256, st.sms);
  if (v4)
    qi32_fixup_kernel<4><<<gv4, 256, 0, stream>>>(cbuf, y, rowterm, colsum, g, q, iq, fq, flag, x, w, fused);
  else
    qi32_fixup_kernel<1><<<gv1, 256, 0, stream>>>(cbuf, y, rowterm, colsum, g, q, iq, fq, flag, x, w, fused);
  rc = check_launch("qi32_fixup_kernel launch");
  if (rc) return rc;
  g_last_path = 11;
  return B200Q_OK;
}

int qi32_common(int qtype, const float* x, const float* w, int32_t* y, const ConvGeom& g, const void* in_qp,
                const void* f_qp, void* stream) {
  if (qtype != B200Q_LINQUANT_U8 && qtype != B200Q_LINQUANT_S5)
    return fail(B200Q_ERR_INVALID_ARG, "quantized conv supports only LinQuantU8 and LinQuantS5");
  if (!in_qp || !f_qp) return fail(B200Q_ERR_INVALID_ARG, "quantized CUDA fprop requires non-null quantization parameters");
  if (!x || !w || !y) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  // Groups of a few channels (depthwise and the like: (c/groups) * (k/groups) <= 16) stay on the
  // direct kernel: a GEMM per group would have 1-4 rows or columns.
  if (g_policy.load() == 0 && static_cast<long long>(g.cg) * g.kg > 16) {
    rc = qi32_tensor_core(*st, qtype, x, w, y, g, in_qp, f_qp, as_stream(stream));
    if (rc != B200Q_ERR_UNSUPPORTED) return rc;
  }
  const int stride = qtype == B200Q_LINQUANT_U8 ? (int)sizeof(b200q_qparams_u8) : (int)sizeof(b200q_qparams_s5);
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  qi32_conv_kernel<<<grid_for(total, 256, st->sms), 256, 0, as_stream(stream)>>>(
      x, w, y, g, static_cast<const uint8_t*>(in_qp), static_cast<const uint8_t*>(f_qp), stride,
      qtype == B200Q_LINQUANT_S5);
  g_last_path = 5;
  return check_launch("qi32_conv_kernel launch");
}

// ------------------------------------------------------------- workspace
// Grow-only scratch per (device, stream), allocated stream-ordered (cudaMallocAsync /
// cudaFreeAsync on that stream), so calls on one stream may reuse it without synchronising and
// calls on different streams never share it.
struct Workspace {
  void* ptr = nullptr;
  size_t cap = 0;
};
std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;
std::mutex g_ws_mu;

int get_workspace(size_t bytes, cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace& w = g_ws[{dev, stream}];
  if (w.cap < bytes) {
    if (w.ptr) {
      e = cudaFreeAsync(w.ptr, stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync(workspace)");
      w.ptr = nullptr;
      w.cap = 0;
    }
    size_t nb = bytes + bytes / 4;
    nb = (nb + (2u << 20) - 1) & ~static_cast<size_t>((2u << 20) - 1);
    e = cudaMallocAsync(&w.ptr, nb, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync(workspace)");
    w.cap = nb;
  }
  *out = w.ptr;
  return B200Q_OK;
}

size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Bytes of scratch the packed low-channel path needs: the im2col matrix then the padded weights.
size_t packed_scratch_bytes(long long rows, int k, int kp) {
  return round256(static_cast<size_t>(rows) * kp) + round256(static_cast<size_t>(k) * kp);
}

// Low-channel conv through scratch: pack im2col rows and zero-padded weights, then run the
// tcgen05 GEMM in tiled mode (M = N*Ho*Wo rows, K = kp, N = output channels).
int run_packed_conv(const DeviceState& st, const int8_t* x, const int8_t* w, void* y, const ConvGeom& g,
                    const Epilogue& e, int8_t* scratch, cudaStream_t stream) {
  const long long rows = static_cast<long long>(g.n) * g.ho * g.wo;
  const int rsc = g.r * g.s * g.c;
  const int kp = (rsc + 31) / 32 * 32;
  int8_t* a_buf = scratch;
  int8_t* w_buf = scratch + round256(static_cast<size_t>(rows) * kp);
  // Short packed rows (kp <= 64: 1x1 convs with C % 16 != 0, the 3x3 C = 3 stem) pack faster one
  // thread per row; long rows (the 7x7 stem, kp = 160) faster through the shared-memory tile.
  if (g_pack_words && g.dil_w == 1 && kp <= 64) {
    const size_t x_bytes = static_cast<size_t>(g.n) * g.h * g.w * g.c;
    im2col_pack_words_kernel<<<grid_for(static_cast<size_t>(rows), 256, st.sms), 256, 0, stream>>>(x, a_buf, g, kp,
                                                                                                  rows, x_bytes);
  } else {
    int tile_rows = 16384 / kp;
    if (tile_rows > 64) tile_rows = 64;
    if (tile_rows < 1) tile_rows = 1;
    const long long blocks_needed = (rows + tile_rows - 1) / tile_rows;
    const int pack_grid = static_cast<int>(blocks_needed < st.sms * 16ll ? blocks_needed : st.sms * 16ll);
    im2col_pack_s8_kernel<<<pack_grid, 256, static_cast<size_t>(tile_rows) * kp, stream>>>(x, a_buf, g, kp, rows,
                                                                                          tile_rows);
  }
  int rc = check_launch("im2col_pack_s8_kernel launch");
  if (rc) return rc;
  weight_pad_s8_kernel<<<grid_for(static_cast<size_t>(g.k) * kp, 256, st.sms), 256, 0, stream>>>(w, w_buf, g.k, rsc,
                                                                                                   kp);
  rc = check_launch("weight_pad_s8_kernel launch");
  if (rc) return rc;
  TcArgs a{};
  a.mode = 0;
  a.BK = kp % 128 == 0 ? 128 : (kp % 64 == 0 ? 64 : 32);
  a.BN = pick_bn(g.k, 0);
  a.M = static_cast<int>(rows);
  a.N = g.k;
  a.batch = 1;
  a.num_kb = kp / a.BK;
  a.epi = e;
  a.out = y;
  a.ldc = g.k;
  a.vec_ok = g.k % 16 == 0;
  CUtensorMap ma, mb;
  rc = encode_tiled_3d(&ma, a_buf, static_cast<uint64_t>(kp), static_cast<uint64_t>(rows), 1, a.BK, kTcBM, a.BK);
  if (rc) return rc;
  a.pair = want_pair(st.sms, a);
  rc = encode_tiled_3d(&mb, w_buf, static_cast<uint64_t>(kp), static_cast<uint64_t>(g.k), 1, a.BK,
                       a.pair ? a.BN / 2 : a.BN, a.BK);
  if (rc) return rc;
  return launch_tc(st, ma, mb, a, stream);
}

// ------------------------------------------------- fixed scratch (no allocation)
// Scratch for b200q_conv2d_s8_packed_noalloc: a file-scope device array, so that entry point never
// allocates.  Every GPU that loads this library holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = 32u << 20;  // 32 MiB
static __device__ __align__(256) int8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device.  In host code the array's name is only a host
// stand-in, so the address is looked up once per device, with that device current.
int8_t* g_noalloc_ptr[64] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(int8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200Q_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = static_cast<int8_t*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return B200Q_OK;
}

// ------------------------------------------------------------------ fp32 (3 x TF32 split) paths
int f32_pack(const DeviceState& st, const float* src, float* dst, const F32Pack& q, cudaStream_t stream) {
  const long long tiles = static_cast<long long>(q.batch) * ((q.rows + 31) / 32) * (q.kp / 32);
  const long long cap = static_cast<long long>(st.sms) * 16;
  const int grid = static_cast<int>(tiles < 1 ? 1 : (tiles < cap ? tiles : cap));
  f32_pack_kernel<<<grid, 256, 0, stream>>>(src, dst, q);
  return check_launch("f32_pack_kernel launch");
}

// C[b][m][n] = sum over the packed reduction of A'[b][m][.] * B'[b][n][.] (3 x kp fp32 per row),
// fp32 accumulators written bit for bit at C + b * bstride + m * ldc + n.
int f32_gemm(const DeviceState& st, const float* ap, const float* bp, float* c, int batch, int M, int N, int kp,
             long long ldc, long long bstride, cudaStream_t stream) {
  TcArgs a{};
  a.mode = 0;
  a.tf32 = 1;
  a.BK = 128;
  a.BN = pick_bn(N, 0);
  a.M = M;
  a.N = N;
  a.batch = batch;
  a.b_batched = batch > 1;
  a.num_kb = 3 * kp / 32;
  a.epi = Epilogue{kOutS32, 0, 0, 0, nullptr, nullptr, nullptr, 0.0f};
  a.out = c;
  a.ldc = ldc;
  a.batch_stride = bstride;
  a.vec_ok = N % 4 == 0 && ldc % 4 == 0 && bstride % 4 == 0 && aligned16(c);
  const uint64_t row_bytes = 12ull * kp;
  CUtensorMap ma, mb;
  int rc = encode_tiled_3d(&ma, ap, row_bytes, static_cast<uint64_t>(M), static_cast<uint64_t>(batch), 128, kTcBM, 128);
  if (rc) return rc;
  rc = encode_tiled_3d(&mb, bp, row_bytes, static_cast<uint64_t>(N), static_cast<uint64_t>(batch), 128, a.BN, 128);
  if (rc) return rc;
  return launch_tc(st, ma, mb, a, stream);
}

F32Pack f32_conv_pack(const ConvGeom& g, int mode, int rows, int cols, int batch, int lo_mask, int chunk) {
  F32Pack q{};
  q.mode = mode;
  q.rows = rows;
  q.cols = cols;
  q.kp = (cols + 31) / 32 * 32;
  q.lo_mask = lo_mask;
  q.batch = batch;
  q.g = g;
  q.T = g.r * g.s * g.cg;
  q.nblk = g.by * g.bx;
  q.mb = g.n * g.bho * g.bwo;
  q.chunk = chunk;
  return q;
}

bool f32_sizes_ok(const ConvGeom& g) {
  const long long mb = static_cast<long long>(g.n) * g.bho * g.bwo;
  const long long T = static_cast<long long>(g.r) * g.s * g.cg;
  return mb < (1ll << 30) && T < (1 << 24) && static_cast<long long>(g.by) * g.bx * g.groups < (1 << 16);
}

// Whether an fp32 conv of this geometry (input x of g.c channels) can run through the im2col TMA:
// no blocks, 16-byte group channel starts and pointers, the im2col corner limits, and at least
// 128 KiB of input (smaller im2col maps take the packed route).  Groups are batch items.
bool f32_im2col_ok(const ConvGeom& g, const void* x, const void* y) {
  const bool corners_ok = g.pad_w <= 127 && g.pad_h <= 127 && g.pad_w - (g.s - 1) * g.dil_w >= -128 &&
                          g.pad_h - (g.r - 1) * g.dil_h >= -128 && (g.s - 1) * g.dil_w <= 255 &&
                          (g.r - 1) * g.dil_h <= 255 && g.stride_h <= 8 && g.stride_w <= 8;
  const long long M = static_cast<long long>(g.n) * g.ho * g.wo;
  const size_t x_bytes = static_cast<size_t>(g.n) * g.h * g.w * g.c * 4;
  return g.by == 1 && g.bx == 1 && g.cg % 4 == 0 && aligned16(x) && aligned16(y) && corners_ok &&
         x_bytes >= (128u << 10) && M < (1ll << 31) && g.k <= 65535;
}

// fp32 conv of x [n,h,w,c] with KRSC weights (flip = 0) or with the data-gradient filter of a
// stride-1 conv (flip = 1, see f32_pack_taps_kernel), written to y [n,ho,wo,k] directly.
int f32_conv_im2col(const DeviceState& st, const float* x, const float* w, float* y, const ConvGeom& g, int flip,
                    cudaStream_t stream) {
  const int cpad = (g.cg + 31) / 32 * 32;
  const int L = g.r * g.s * cpad;
  const size_t x_elems = static_cast<size_t>(g.n) * g.h * g.w * g.c;
  const size_t x_bytes = round256(x_elems * 4);
  const size_t b_bytes = round256(static_cast<size_t>(g.k) * 3 * L * 4);
  void* ws = nullptr;
  int rc = get_workspace(2 * x_bytes + b_bytes, stream, &ws);
  if (rc) return rc;
  float* xhi = static_cast<float*>(ws);
  float* xlo = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + x_bytes);
  float* bp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + 2 * x_bytes);
  f32_split_kernel<<<grid_for(x_elems / 4, 256, st.sms), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(xhi), reinterpret_cast<float4*>(xlo), x_elems / 4);
  if ((rc = check_launch("f32_split_kernel launch"))) return rc;
  f32_pack_taps_kernel<<<grid_for(static_cast<size_t>(g.k) * 3 * L, 256, st.sms), 256, 0, stream>>>(
      w, bp, g.k, g.r, g.s, g.cg, cpad, flip, g.kg);
  if ((rc = check_launch("f32_pack_taps_kernel launch"))) return rc;
  TcArgs a{};
  a.mode = 1;
  a.tf32 = 1;
  a.BK = 128;
  a.cchunks = cpad / 32;
  a.kb_third = g.r * g.s * a.cchunks;
  a.num_kb = 3 * a.kb_third;
  a.BN = pick_bn(g.kg, 0);
  a.M = g.n * g.ho * g.wo;
  a.N = g.kg;
  a.batch = g.groups;  // group b: channels from b * cg, filter rows b * kg.., output columns b * kg..
  a.b_batched = g.groups > 1;
  a.grp_bytes = 4 * g.cg;
  a.batch_stride = g.kg;
  a.epi = Epilogue{kOutS32, 0, 0, 0, nullptr, nullptr, nullptr, 0.0f};
  a.out = y;
  a.ldc = g.k;
  a.vec_ok = g.kg % 4 == 0 && g.k % 4 == 0;
  a.Ho = g.ho; a.Wo = g.wo; a.S = g.s;
  a.stride_h = g.stride_h; a.stride_w = g.stride_w;
  a.pad_h = g.pad_h; a.pad_w = g.pad_w;
  a.dil_h = g.dil_h; a.dil_w = g.dil_w;
  // the fp32 tensor as bytes: 4 * c byte channels per pixel, 128-byte (32-float) channel boxes
  ConvGeom gb = g;
  gb.c = 4 * g.c;
  CUtensorMap ma, ma2, mb;
  if ((rc = encode_im2col(&ma, reinterpret_cast<const int8_t*>(xhi), gb, 128))) return rc;
  if ((rc = encode_im2col(&ma2, reinterpret_cast<const int8_t*>(xlo), gb, 128))) return rc;
  if ((rc = encode_tiled_3d(&mb, bp, 12ull * L, static_cast<uint64_t>(g.kg), static_cast<uint64_t>(g.groups), 128,
                            a.BN, 128)))
    return rc;
  if ((rc = launch_tc(st, ma, mb, a, stream, &ma2))) return rc;
  g_last_path = 13;
  return B200Q_OK;
}

int f32_fprop(const DeviceState& st, const float* x, const float* w, const float* bias, int bias_mode, float* y,
              const ConvGeom& g, cudaStream_t stream) {
  if (!bias && f32_im2col_ok(g, x, y)) return f32_conv_im2col(st, x, w, y, g, 0, stream);
  const int G = g.groups, nblk = g.by * g.bx, Gp = nblk * G;
  const int mb = g.n * g.bho * g.bwo, T = g.r * g.s * g.cg;
  const F32Pack qa = f32_conv_pack(g, kPackIm2colRows, mb, T, Gp, 4, mb);
  const F32Pack qb = f32_conv_pack(g, kPackWRows, g.kg, T, Gp, 2, mb);
  // Without blocks or bias the GEMM writes y directly: row m of group grp at y + m * K + grp * Kg.
  const bool direct = nblk == 1 && !bias;
  const size_t a_bytes = round256(static_cast<size_t>(Gp) * mb * 3 * qa.kp * 4);
  const size_t b_bytes = round256(static_cast<size_t>(Gp) * g.kg * 3 * qb.kp * 4);
  const size_t c_bytes = direct ? 0 : round256(static_cast<size_t>(Gp) * mb * g.kg * 4);
  void* ws = nullptr;
  int rc = get_workspace(a_bytes + b_bytes + c_bytes, stream, &ws);
  if (rc) return rc;
  float* ap = static_cast<float*>(ws);
  float* bp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes);
  float* cp = direct ? y : reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes + b_bytes);
  if ((rc = f32_pack(st, x, ap, qa, stream))) return rc;
  if ((rc = f32_pack(st, w, bp, qb, stream))) return rc;
  if (direct)
    rc = f32_gemm(st, ap, bp, cp, G, mb, g.kg, qa.kp, g.k, g.kg, stream);
  else
    rc = f32_gemm(st, ap, bp, cp, Gp, mb, g.kg, qa.kp, g.kg, static_cast<long long>(mb) * g.kg, stream);
  if (rc) return rc;
  if (!direct) {
    const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
    f32_fprop_scatter_kernel<<<grid_for(total, 256, st.sms), 256, 0, stream>>>(cp, y, g, mb, bias, bias_mode);
    if ((rc = check_launch("f32_fprop_scatter_kernel launch"))) return rc;
  }
  g_last_path = 13;
  return B200Q_OK;
}

int f32_bprop(const DeviceState& st, const float* dy, const float* w, float* dx, const ConvGeom& g,
              cudaStream_t stream) {
  // Stride 1: dx is the conv of dy with the flipped, transposed filter and padding dil * (R - 1) - pad.
  if (g.stride_h == 1 && g.stride_w == 1 && g.by == 1 && g.bx == 1) {
    ConvGeom gb = g;
    gb.h = g.ho; gb.w = g.wo; gb.c = g.k;
    gb.ho = g.h; gb.wo = g.w; gb.k = g.c;
    gb.pad_h = g.dil_h * (g.r - 1) - g.pad_h;
    gb.pad_w = g.dil_w * (g.s - 1) - g.pad_w;
    gb.cg = g.kg; gb.kg = g.cg; gb.bho = gb.ho; gb.bwo = gb.wo;
    if (gb.pad_h >= 0 && gb.pad_w >= 0 && f32_im2col_ok(gb, dy, dx)) return f32_conv_im2col(st, dy, w, dx, gb, 1, stream);
  }
  const int G = g.groups, nblk = g.by * g.bx, Gp = nblk * G;
  const int mb = g.n * g.bho * g.bwo, T = g.r * g.s * g.cg;
  const F32Pack qa = f32_conv_pack(g, kPackDyRows, mb, g.kg, Gp, 4, mb);
  const F32Pack qb = f32_conv_pack(g, kPackWCols, T, g.kg, Gp, 2, mb);
  const size_t a_bytes = round256(static_cast<size_t>(Gp) * mb * 3 * qa.kp * 4);
  const size_t b_bytes = round256(static_cast<size_t>(Gp) * T * 3 * qb.kp * 4);
  const size_t c_bytes = round256(static_cast<size_t>(Gp) * mb * T * 4);
  void* ws = nullptr;
  int rc = get_workspace(a_bytes + b_bytes + c_bytes, stream, &ws);
  if (rc) return rc;
  float* ap = static_cast<float*>(ws);
  float* bp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes);
  float* col = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes + b_bytes);
  if ((rc = f32_pack(st, dy, ap, qa, stream))) return rc;
  if ((rc = f32_pack(st, w, bp, qb, stream))) return rc;
  if ((rc = f32_gemm(st, ap, bp, col, Gp, mb, T, qa.kp, T, static_cast<long long>(mb) * T, stream))) return rc;
  const size_t total = static_cast<size_t>(g.n) * g.h * g.w * g.c;
  f32_col2im_kernel<<<grid_for(total, 256, st.sms), 256, 0, stream>>>(col, dx, g, mb, T);
  if ((rc = check_launch("f32_col2im_kernel launch"))) return rc;
  g_last_path = 13;
  return B200Q_OK;
}

int f32_grad(const DeviceState& st, const float* x, const float* dy, float* dw, float* dbias, int bias_mode,
             const ConvGeom& g, cudaStream_t stream) {
  const int G = g.groups, nblk = g.by * g.bx, Gp = nblk * G;
  const int mb = g.n * g.bho * g.bwo, T = g.r * g.s * g.cg;
  // The reduction runs over the block's output pixels: split it so that every SM has output tiles.
  const long long tiles = static_cast<long long>(Gp) * ((g.kg + kTcBM - 1) / kTcBM) * ((T + 255) / 256);
  long long splits = (2ll * st.sms + tiles - 1) / tiles;
  const long long max_splits = (mb + 511) / 512;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  const int chunk = static_cast<int>(((mb + splits - 1) / splits + 31) / 32 * 32);
  splits = (mb + chunk - 1) / chunk;
  const int bt = static_cast<int>(splits) * Gp;
  const F32Pack qa = f32_conv_pack(g, kPackDyCols, g.kg, chunk, bt, 4, chunk);
  const F32Pack qb = f32_conv_pack(g, kPackIm2colCols, T, chunk, bt, 2, chunk);
  const size_t a_bytes = round256(static_cast<size_t>(bt) * g.kg * 3 * qa.kp * 4);
  const size_t b_bytes = round256(static_cast<size_t>(bt) * T * 3 * qb.kp * 4);
  const size_t c_bytes = round256(static_cast<size_t>(bt) * g.kg * T * 4);
  void* ws = nullptr;
  int rc = get_workspace(a_bytes + b_bytes + c_bytes, stream, &ws);
  if (rc) return rc;
  float* ap = static_cast<float*>(ws);
  float* bp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes);
  float* cp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes + b_bytes);
  if ((rc = f32_pack(st, dy, ap, qa, stream))) return rc;
  if ((rc = f32_pack(st, x, bp, qb, stream))) return rc;
  if ((rc = f32_gemm(st, ap, bp, cp, bt, g.kg, T, qa.kp, T, static_cast<long long>(g.kg) * T, stream))) return rc;
  const size_t total = static_cast<size_t>(g.k) * nblk * T;
  f32_grad_reduce_kernel<<<grid_for(total, 256, st.sms), 256, 0, stream>>>(cp, dw, g, nblk, T,
                                                                           static_cast<int>(splits));
  if ((rc = check_launch("f32_grad_reduce_kernel launch"))) return rc;
  if (dbias) {
    const int entries = g.k * nblk;
    f32_dbias_kernel<<<entries < st.sms * 8 ? entries : st.sms * 8, 256, 0, stream>>>(dy, dbias, g, bias_mode);
    if ((rc = check_launch("f32_dbias_kernel launch"))) return rc;
  }
  g_last_path = 13;
  return B200Q_OK;
}

}  // namespace
}  // namespace b200q

using namespace b200q;

extern "C" {

const char* b200q_last_error(void) { return g_errmsg; }
int b200q_last_path(void) { return g_last_path; }
void b200q_set_path_policy(int policy) { g_policy.store(policy); }
long long b200q_tc_launch_count(void) { return g_tc_launches.load(); }

int b200q_conv_out_shape(int h, int w, int c, int r, int s, int k, const b200q_conv_params* p, int* ho, int* wo) {
  if (!p || !ho || !wo) return fail(B200Q_ERR_INVALID_ARG, "null argument");
  if (p->groups <= 0) return fail(B200Q_ERR_INVALID_ARG, "groups must be > 0");
  if (c % p->groups != 0) return fail(B200Q_ERR_INVALID_ARG, "input channels must be divisible by groups");
  if (k % p->groups != 0) return fail(B200Q_ERR_INVALID_ARG, "output channels must be divisible by groups");
  const int hn = h + 2 * p->pad_h - p->dilation_h * (r - 1) - 1;
  const int wn = w + 2 * p->pad_w - p->dilation_w * (s - 1) - 1;
  if (hn < 0 || wn < 0) return fail(B200Q_ERR_INVALID_ARG, "invalid output size (negative numerator)");
  if (p->stride_h <= 0 || p->stride_w <= 0) return fail(B200Q_ERR_INVALID_ARG, "stride must be > 0");
  *ho = hn / p->stride_h + 1;
  *wo = wn / p->stride_w + 1;
  if (*ho <= 0 || *wo <= 0) return fail(B200Q_ERR_INVALID_ARG, "computed output size is <= 0");
  return B200Q_OK;
}

int b200q_fprop_nhwc_qi32(int qtype, const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w, int c,
                          int r, int s, int k, const b200q_conv_params* p, const void* d_in_qp, const void* d_f_qp,
                          void* stream) {
  ConvGeom g;
  int rc = conv_geom(n, h, w, c, r, s, k, p, 1, 1, &g);
  if (rc) return rc;
  return qi32_common(qtype, d_x, d_w, d_y, g, d_in_qp, d_f_qp, stream);
}

int b200q_block_fprop_nhwc_qi32(int qtype, const float* d_x, const float* d_w, int32_t* d_y, int n, int h, int w,
                                int c, int r, int s, int k, const b200q_conv_params* p, int block_by, int block_bx,
                                const void* d_in_qp, const void* d_f_qp, void* stream) {
  ConvGeom g;
  int rc = conv_geom(n, h, w, c, r, s, k, p, block_by, block_bx, &g);
  if (rc) return rc;
  return qi32_common(qtype, d_x, d_w, d_y, g, d_in_qp, d_f_qp, stream);
}

// tcgen05 batched GEMM over int8 operands in bmm.h's layouts (shapes checked by the caller:
// 16-byte aligned pointers, the contiguous dimensions of A and B multiples of 16).
static int bmm_s8_tcgen05(DeviceState& st, const int8_t* A, const int8_t* B, void* C, int batch, int M, int N,
                          int K, bool ta, bool tb, const Epilogue& e, cudaStream_t cs) {
  int rc = 0;
  TcArgs a{};
  a.mode = 0;
  a.BK = 128;
  a.a_major = ta ? 1 : 0;
  a.b_major = tb ? 0 : 1;  // B stored [K][N] (no transpose) is N-contiguous = MN-major
  a.BN = pick_bn(N, a.b_major);
  a.M = M;
  a.N = N;
  a.batch = batch;
  a.b_batched = 1;
  a.num_kb = (K + a.BK - 1) / a.BK;
  a.epi = e;
  a.out = C;
  a.ldc = N;
  a.batch_stride = static_cast<long long>(M) * N;
  a.vec_ok = N % 16 == 0;
  CUtensorMap ma, mb;
  if (!ta)
    rc = encode_tiled_3d(&ma, A, (uint64_t)K, (uint64_t)M, (uint64_t)batch, a.BK, kTcBM, 128);
  else
    rc = encode_tiled_3d(&ma, A, (uint64_t)M, (uint64_t)K, (uint64_t)batch, kTcBM, a.BK, 128);
  if (rc) return rc;
  a.pair = want_pair(st.sms, a);
  if (tb)
    rc = encode_tiled_3d(&mb, B, (uint64_t)K, (uint64_t)N, (uint64_t)batch, a.BK, a.pair ? a.BN / 2 : a.BN, 128);
  else
    rc = encode_tiled_3d(&mb, B, (uint64_t)N, (uint64_t)K, (uint64_t)batch, 128, a.BK, 128);
  if (rc) return rc;
  g_last_path = a.pair ? 8 : 2;
  return launch_tc(st, ma, mb, a, cs);
}

int b200q_bmm_matmul_i32(const int32_t* A, const int32_t* B, int32_t* C, int batch, int M, int N, int K,
                         int trans_a, int trans_b, void* stream) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(B200Q_ERR_INVALID_ARG, "negative bmm dimension");
  if (batch == 0 || M == 0 || N == 0) return B200Q_OK;
  if (!A || !B || !C) return fail(B200Q_ERR_INVALID_ARG, "null bmm pointer");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  Epilogue e{kOutS32, 0, 0, 0, nullptr, nullptr};
  cudaStream_t cs = as_stream(stream);
  // Tensor-core route: operands whose values all fit int8 give the same C from an int8 GEMM with
  // int32 accumulation (|a*b| <= 2^14, so sums of K <= 2^17 - 1 products cannot wrap).  The operands
  // are copied to int8 on the device; a value outside [-128, 127] sets a flag, and the CUDA-core
  // kernel below then runs (every block reads the flag and returns at once while it is clear).
  const int* run_if = nullptr;
  int run_gen = 0;
  const bool ta = trans_a != 0, tb = trans_b != 0;
  if (g_policy.load() == 0 && K > 0 && K < (1 << 17) && aligned16(A) && aligned16(B) && aligned16(C) &&
      (ta ? M % 16 == 0 : K % 16 == 0) && (tb ? K % 16 == 0 : N % 16 == 0)) {
    const size_t na = static_cast<size_t>(batch) * M * K, nb_ = static_cast<size_t>(batch) * K * N;
    const size_t a_bytes = round256(na), b_bytes = round256(nb_);
    void* ws = nullptr;
    rc = get_workspace(a_bytes + b_bytes + 256, cs, &ws);
    if (rc) return rc;
    int8_t* a8 = static_cast<int8_t*>(ws);
    int8_t* b8 = a8 + a_bytes;
    int* flag = reinterpret_cast<int*>(b8 + b_bytes);
    run_gen = next_flag_gen();  // the flag is not cleared: the kernels compare it with this number
    i32_to_s8_kernel<<<grid_for((na + nb_) / 16, 256, st->sms), 256, 0, cs>>>(A, a8, na, B, b8, nb_, flag, run_gen);
    rc = check_launch("i32_to_s8_kernel launch");
    if (rc) return rc;
    rc = bmm_s8_tcgen05(*st, a8, b8, C, batch, M, N, K, ta, tb, e, cs);
    if (rc) return rc;
    run_if = flag;
  }
  {
    // one block per 64 x 64 tile; the gated fallback after the tensor-core route launches one block
    // per SM instead (the blocks walk the tiles), so it costs one small launch while its flag is clear
    const long long tiles = static_cast<long long>((N + 63) / 64) * ((M + 63) / 64) * batch;
    const long long cap = run_if ? st->sms : 0x7fffffffll;
    const int blocks = static_cast<int>(tiles < cap ? tiles : cap);
    bmm_simt_kernel<int32_t><<<blocks, 256, 0, cs>>>(A, B, C, M, N, K, ta, tb, e, run_if, run_gen, batch);
    rc = check_launch("bmm_simt_kernel<int32> launch");
    if (rc) return rc;
  }
  g_last_path = run_if ? 16 : 6;
  return B200Q_OK;
}

// Tile plan of dw_tma_s8_kernel for a 3x3 depthwise conv of stride 1 or 2 (see dw_tma.cuh);
// false when the geometry does not fit the kernel's limits (TMA boxes of at most 256 per dimension).
static bool dw_tma_plan(const ConvGeom& g, DwPlan* out) {
  DwPlan p{};
  const int s = g.stride_h;
  if (g.c <= 256) {
    p.CB = g.c;
  } else {
    p.CB = 16;
    for (int d = 16; d >= 1; --d)
      if ((g.c / 16) % d == 0) {
        p.CB = 16 * d;
        break;
      }
  }
  p.g8 = p.CB / 8;
  const int max_cols = 256 / p.g8;
  p.col_tiles = (g.wo + max_cols - 1) / max_cols;
  for (;;) {
    p.TW = (g.wo + p.col_tiles - 1) / p.col_tiles;
    p.wbox = (p.TW - 1) * s + 3;
    if (p.wbox <= 256) break;
    ++p.col_tiles;
  }
  p.RG = 256 / (p.g8 * p.TW);
  if (p.RG < 1) return false;
  if (p.RG > g.ho) p.RG = g.ho;
  // rows per thread: the largest count whose box stays within 32 KiB and 256 rows, at most enough
  // to cover the image
  p.rpt = (g.ho + p.RG - 1) / p.RG;
  for (;; --p.rpt) {
    if (p.rpt < 1) return false;
    p.TH = p.RG * p.rpt;
    p.rows_in = (p.TH - 1) * s + 3;
    p.box_bytes = p.CB * p.wbox * p.rows_in;
    if (p.rows_in <= 256 && p.box_bytes <= 32 * 1024) break;
  }
  p.stage = (p.box_bytes + 1023) / 1024 * 1024;
  p.stages = 3;
  p.slabs = g.c / p.CB;
  p.row_tiles = (g.ho + p.TH - 1) / p.TH;
  const long long total = static_cast<long long>(p.slabs) * g.n * p.row_tiles * p.col_tiles;
  if (total >= (1ll << 31)) return false;
  p.total = static_cast<int>(total);
  *out = p;
  return true;
}

static bool dw_tma_ok(const ConvGeom& g, int r, int s, int k, int c, bool has_res, int out_kind) {
  DwPlan p;
  return !has_res && out_kind == kOutS8 && g.groups == c && k == c && c % 16 == 0 && r == 3 && s == 3 &&
         g.dil_h == 1 && g.dil_w == 1 && g.stride_h == g.stride_w && (g.stride_h == 1 || g.stride_h == 2) &&
         dw_tma_plan(g, &p);
}

// Depthwise input map: x as [N][H][W][C] uint8, box {CB, wbox, rows_in, 1}, no swizzle.
static int encode_dw(CUtensorMap* map, const int8_t* x, const ConvGeom& g, const DwPlan& p) {
  cuuint64_t dims[4] = {(cuuint64_t)g.c, (cuuint64_t)g.w, (cuuint64_t)g.h, (cuuint64_t)g.n};
  cuuint64_t strides[3] = {(cuuint64_t)g.c, (cuuint64_t)g.c * g.w, (cuuint64_t)g.c * g.w * g.h};
  cuuint32_t box[4] = {(cuuint32_t)p.CB, (cuuint32_t)p.wbox, (cuuint32_t)p.rows_in, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t*>(x), dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200Q_ERR_CUDA, "cuTensorMapEncodeTiled (depthwise tile) failed (%d)", (int)r);
  return B200Q_OK;
}

// Dispatch of the int8 conv (shared by the plain and the residual-add entry points).
// Kernel family of a conv2d_s8 call (b200q_last_path codes), decided from the geometry, the
// epilogue, pointer alignment and the SM count only, so that b200q_conv2d_s8_plan can predict it
// without a GPU.  conv2d_s8_impl dispatches on the same decision.
struct ConvRoute {
  int path;            // 10 s2d row tiles, 9 row tiles, 2 tiled, 1 im2col, 8 tiled 2-SM, 7 packed, 4 depthwise, 3 generic
  int s2d_r2, s2d_s2;  // path 10: taps of the stride-1 filter over the 2x2-block copy
  int tc_bk;           // paths 1 / 2 / 8: K block bytes per ring stage
  int group;           // path 15: pixels per GEMM row
};

// Pixel grouping of a 1x1 conv (path 15): the largest G in {16, 8, 4, 2} with G * K <= 256,
// G * C <= 256, G * C a multiple of 16 (TMA rows) and M % G == 0; 1 when none fits.
static const bool g_group1x1 = [] {
  const char* v = getenv("B200Q_GROUP1X1");
  return !(v && v[0] == '0');
}();
static int pick_group(int c, int k, long long M) {
  for (int G : {16, 8, 4, 2})
    if (G * k <= 256 && G * c <= 256 && (G * c) % 16 == 0 && M % G == 0) return G;
  return 1;
}

static int tc_pick_bk(int c) {
  // The K block (128 / 64 / 32 bytes of channels per ring stage) with the fewest blocks per tap,
  // ties to the smaller block; TMA zero-fills the channels past C.  Short reductions are bound by
  // the TMA's per-row requests, not by the MMAs: C = 96 at 128-byte blocks (one per pixel row
  // instead of three 32-byte ones) runs a 96 -> 24 1x1 conv in 0.028 ms instead of 0.046.
  int best = 32;
  for (int bk : {64, 128})
    if ((c + bk - 1) / bk < (c + best - 1) / best) best = bk;
  return best;
}

static ConvRoute route_conv_s8(const ConvGeom& g, int h, int w, int c, int r, int s, int k, bool x_aligned,
                               bool w_aligned, bool y_aligned, bool epi_aligned, bool has_res, int out_kind, int sms) {
  const bool out_aligned = y_aligned && epi_aligned;
  (void)h;
  (void)w;
  ConvRoute rt{3, 0, 0, 0, 0};
  const bool auto_policy = g_policy.load() == 0;
  const long long M = static_cast<long long>(g.n) * g.ho * g.wo;
  const size_t x_bytes = static_cast<size_t>(g.n) * g.h * g.w * c;
  const bool vec_ptrs = x_aligned && w_aligned && out_aligned;
  const bool is_1x1_plain = r == 1 && s == 1 && g.stride_h == 1 && g.stride_w == 1 && g.pad_h == 0 && g.pad_w == 0;
  const bool corners_ok = g.pad_w <= 127 && g.pad_h <= 127 && g.pad_w - (s - 1) * g.dil_w >= -128 &&
                          g.pad_h - (r - 1) * g.dil_h >= -128 && (s - 1) * g.dil_w <= 255 && (r - 1) * g.dil_h <= 255 &&
                          g.stride_h <= 8 && g.stride_w <= 8;
  // Space-to-depth row tiles for stride-2 convs of 1-4 channels (network stems).
  if (g_s2d && auto_policy && g.groups == 1 && g.stride_h == 2 && g.stride_w == 2 && g.dil_h == 1 && g.dil_w == 1 &&
      c >= 1 && c <= 4 && k <= 256 && M >= 1024 && M < (1ll << 31) && out_aligned && g.ho > 0 && g.wo > 0) {
    auto fdiv2 = [](int v) { return v >= 0 ? v / 2 : -((1 - v) / 2); };
    const int yoff = -((g.pad_h + 1) / 2), xoff = -((g.pad_w + 1) / 2);
    const int r2 = fdiv2(r - 1 - g.pad_h) - yoff + 1;
    const int s2 = (fdiv2(s - 1 - g.pad_w) - xoff + 1 + 1) / 2 * 2;
    if (r2 >= 2 && r2 <= 4 && (s2 == 2 || s2 == 4) && g.wo + s2 - 1 <= 128) {
      rt.path = 10;
      rt.s2d_r2 = r2;
      rt.s2d_s2 = s2;
      return rt;
    }
  }
  // Row tiles for 3x3 / stride 1 / pad 1 convs whose weights stay resident beside two window stages.
  {
    const int rt_P = g.wo + 1;
    const int rt_bn = pick_bn(k, 0);
    const long long rt_T0 = rt_P <= 128 ? 128 / rt_P : 1;
    const long long rt_stage0 = ((rt_T0 + 3) * rt_P * c + (2 * rt_P + 2 + 128) * 16 + 1023) / 1024 * 1024;
    const bool rt_fits = 9ll * c * rt_bn + 2 * rt_stage0 + kSmemReserve + 8 * 1024 <= kSmemLimit;
    if (g_rowtile && auto_policy && g.groups == 1 && r == 3 && s == 3 && g.stride_h == 1 && g.stride_w == 1 &&
        g.pad_h == 1 && g.pad_w == 1 && g.dil_h == 1 && g.dil_w == 1 && (c == 32 || c == 64 || c == 128) &&
        k <= 256 && rt_P <= 128 && rt_fits && vec_ptrs && M < (1ll << 31)) {
      rt.path = 9;
      return rt;
    }
  }
  // Pixel-grouped 1x1 GEMM for narrow layers (G * K <= 256 and G * C <= 256: one N tile, resident
  // block-diagonal weights): G times the outputs per tile, and TMA rows of G * C bytes.
  if (g_group1x1 && auto_policy && g.groups == 1 && is_1x1_plain && vec_ptrs && M < (1ll << 31)) {
    const int G = pick_group(c, k, M);
    if (G > 1) {
      rt.path = 15;
      rt.group = G;
      rt.tc_bk = tc_pick_bk(G * c);
      return rt;
    }
  }
  // tcgen05 tiled (1x1 / s1 / p0) or im2col: C % 16 == 0; im2col only for activations of at least
  // 128 KiB (a driver limitation on small im2col maps).
  if (auto_policy && g.groups == 1 && c % 16 == 0 && vec_ptrs && M < (1ll << 31) &&
      (is_1x1_plain || (corners_ok && x_bytes >= (128u << 10)))) {
    rt.tc_bk = tc_pick_bk(c);
    rt.path = is_1x1_plain ? 2 : 1;
    if (is_1x1_plain) {
      TcArgs a{};
      a.mode = 0;
      a.BK = rt.tc_bk;
      a.BN = pick_bn(k, 0);
      a.M = static_cast<int>(M);
      a.N = k;
      a.batch = 1;
      a.conv_b = c % a.BK != 0;
      a.num_kb = (c + a.BK - 1) / a.BK;
      a.epi.out_kind = out_kind;
      if (want_pair(sms, a)) rt.path = 8;
    }
    return rt;
  }
  // Low-channel / small convs: im2col pack into the stream's workspace, then tcgen05.
  const int kp_packed = (r * s * c + 31) / 32 * 32;
  if (auto_policy && g.groups == 1 && (c % 16 != 0 ? M >= 4096 : M >= 64) && M < (1ll << 31) && kp_packed <= 16384 &&
      out_aligned) {
    rt.path = 7;
    return rt;
  }
  if (g_dw_tma && auto_policy && x_aligned && y_aligned && dw_tma_ok(g, r, s, k, c, has_res, out_kind)) {
    rt.path = 12;
    return rt;
  }
  if (!has_res && g.groups == c && k == c && c % 8 == 0 && c <= 8 * 256 && r == 3 && s == 3 && M < (1ll << 31) &&
      x_aligned && y_aligned) {
    rt.path = 4;
    return rt;
  }
  return rt;
}

static int conv2d_s8_impl(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias, const float* d_scale,
                   const int8_t* d_res, float res_scale, void* d_y, int n, int h, int w, int c, int r, int s, int k,
                   const b200q_conv_params* p, const b200q_epilogue* epi, void* stream) {
  ConvGeom g;
  int rc = conv_geom(n, h, w, c, r, s, k, p, 1, 1, &g);
  if (rc) return rc;
  if (!d_x || !d_w || !d_y) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  Epilogue e{};
  rc = make_epilogue(epi, d_bias, d_scale, &e);
  if (rc) return rc;
  if (d_res) {
    if (e.out_kind != kOutS8) return fail(B200Q_ERR_INVALID_ARG, "a residual add needs int8 outputs");
    e.res = d_res;
    e.res_scale = res_scale;
  }
  DeviceState* st = nullptr;
  rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t cs = as_stream(stream);
  const long long M = static_cast<long long>(n) * g.ho * g.wo;
  const bool is_1x1_plain = r == 1 && s == 1 && g.stride_h == 1 && g.stride_w == 1 && g.pad_h == 0 && g.pad_w == 0;
  const bool epi_aligned = (!d_bias || aligned16(d_bias)) && (!d_scale || aligned16(d_scale)) &&
                           (!d_res || aligned16(d_res));
  const ConvRoute route = route_conv_s8(g, h, w, c, r, s, k, aligned16(d_x), aligned16(d_w), aligned16(d_y),
                                        epi_aligned, d_res != nullptr, e.out_kind, st->sms);
  // Space-to-depth row tiles for stride-2 convs of 1-4 channels (network stems): the input is
  // rearranged into 16-channel pixels of 2x2 blocks, the weights into an R2 x S2 stride-1 filter
  // (S2 even: each K = 32 MMA slice covers two taps), and the conv runs as row tiles over it.
  // Replaces the im2col pack of the low-channel path: the rearranged input is 16/(4C) times the
  // input instead of R*S*C/C times.
  if (route.path == 10) {
    const int yoff = -((g.pad_h + 1) / 2), xoff = -((g.pad_w + 1) / 2);
    const int r2 = route.s2d_r2, s2 = route.s2d_s2;
    const int P = g.wo + s2 - 1;
    // 32-column tiles for stems of at most 32 output channels (twice the row groups in tensor memory)
    const int bn = (k <= 32 && g_rt_groups > 4) ? 32 : pick_bn(k, 0);
    {
      const int h2 = (h + 1) / 2, w2 = (w + 1) / 2;
      const size_t xs_bytes = (static_cast<size_t>(n) * h2 * w2 * 16 + 1023) / 1024 * 1024;
      const size_t ws_bytes = static_cast<size_t>(k) * r2 * s2 * 16;
      void* ws = nullptr;
      rc = get_workspace(xs_bytes + ws_bytes, cs, &ws);
      if (rc) return rc;
      int8_t* xs = static_cast<int8_t*>(ws);
      int8_t* wsd = xs + xs_bytes;
      const size_t px = static_cast<size_t>(n) * h2 * w2;
      const int grid = grid_for(px, 256, st->sms);
      if (c == 1) s2d_s8_kernel<1><<<grid, 256, 0, cs>>>(d_x, xs, n, h, w, h2, w2);
      else if (c == 2) s2d_s8_kernel<2><<<grid, 256, 0, cs>>>(d_x, xs, n, h, w, h2, w2);
      else if (c == 3) s2d_s8_kernel<3><<<grid, 256, 0, cs>>>(d_x, xs, n, h, w, h2, w2);
      else s2d_s8_kernel<4><<<grid, 256, 0, cs>>>(d_x, xs, n, h, w, h2, w2);
      rc = check_launch("s2d_s8_kernel launch");
      if (rc) return rc;
      s2d_weight_s8_kernel<<<grid_for(ws_bytes, 256, st->sms), 256, 0, cs>>>(d_w, wsd, k, r, s, c, r2, s2, g.pad_h,
                                                                             g.pad_w);
      rc = check_launch("s2d_weight_s8_kernel launch");
      if (rc) return rc;
      TcArgs a{};
      a.mode = 2;
      a.rt_pairs = 1;
      a.rt_R = r2;
      a.rt_S = s2;
      a.BK = 32;
      a.cchunks = 1;
      a.num_kb = r2 * s2 / 2;
      a.BN = bn;
      a.M = static_cast<int>(M);
      a.N = k;
      a.batch = 1;
      a.epi = e;
      a.out = d_y;
      a.ldc = k;
      a.vec_ok = k % 16 == 0;
      a.Ho = g.ho; a.Wo = g.wo; a.S = s2;
      a.n_img = n;
      a.rt_P = P;
      a.rt_T = 128 / P;
      a.rt_x0 = xoff;
      a.rt_y0 = yoff;
      a.rt_plane = 16;  // K-direction core-matrix stride: one pixel
      // Row groups: up to g_rt_groups groups of rt_T output rows per tile (one window, one TMEM
      // buffer of BN columns per group, two buffers in tensor memory).
      a.rt_G = g_rt_groups;
      if (a.rt_G > 256 / bn) a.rt_G = 256 / bn;
      const int row_blocks = (g.ho + a.rt_T - 1) / a.rt_T;
      if (a.rt_G > row_blocks) a.rt_G = row_blocks;
      // keep at least one tile per SM
      while (a.rt_G > 1 && static_cast<long long>(n) * ((g.ho + a.rt_T * a.rt_G - 1) / (a.rt_T * a.rt_G)) < st->sms)
        --a.rt_G;
      if (a.rt_G < 1) a.rt_G = 1;
      // Window rows: the last tap slice of the last group's last accumulator row reads pixel
      // (rt_G - 1) * rt_T * P + (r2 - 1) * P + s2 - 1 + 127, which must stay inside the box.
      const int rows = ((a.rt_G - 1) * a.rt_T * P + (r2 - 1) * P + s2 - 1 + 128 + P - 1) / P;
      a.rt_box = rows * P * 16;
      a.rt_stage = (a.rt_box + 1023) / 1024 * 1024;
      CUtensorMap ma, mb;
      rc = encode_tiled_3d(&mb, wsd, static_cast<uint64_t>(r2 * s2 * 16), static_cast<uint64_t>(k), 1, 32, a.BN, 32);
      if (rc) return rc;
      a.rt_wide = 1;
      rc = encode_rowtile_wide(&ma, xs, n, h2, w2, P, rows);
      if (rc) return rc;
      g_last_path = 10;
      return launch_tc(*st, ma, mb, a, cs);
    }
  }
  // Row tiles for 3x3 / stride 1 / pad 1 convs whose weights stay resident: one window load per
  // tile serves all nine taps (the im2col mode loads the window nine times, one row per pixel).
  const int rt_P = g.wo + 1;
  const int rt_bn = pick_bn(k, 0);
  if (route.path == 9) {
    TcArgs a{};
    a.mode = 2;
    a.BK = c;
    a.cchunks = 1;
    a.num_kb = 9;
    a.BN = rt_bn;
    a.M = static_cast<int>(M);
    a.N = k;
    a.batch = 1;
    a.epi = e;
    a.out = d_y;
    a.ldc = k;
    a.vec_ok = k % 16 == 0;
    a.Ho = g.ho; a.Wo = g.wo; a.S = 3;
    a.n_img = n;
    a.rt_P = rt_P;
    a.rt_T = 128 / rt_P;
    a.rt_x0 = -1;
    a.rt_y0 = -1;
    // Row groups: as many groups of rt_T rows as keep two accumulator buffers in tensor memory and
    // the resident weights plus two window stages in shared memory.
    {
      const int max_g = g_rt_groups < 256 / a.BN ? g_rt_groups : 256 / a.BN;
      const int row_blocks = (g.ho + a.rt_T - 1) / a.rt_T;
      a.rt_G = 1;
      for (int gg = max_g < row_blocks ? max_g : row_blocks; gg > 1; --gg) {
        // keep at least one tile per SM (BASELINE config 1 is a single image: 28 tiles of 2 rows)
        if (static_cast<long long>(n) * ((g.ho + a.rt_T * gg - 1) / (a.rt_T * gg)) < st->sms) continue;
        const long long stage = ((a.rt_T * gg + 3) * static_cast<long long>(rt_P) * c + (2 * rt_P + 2 + 128) * 16 +
                                 1023) / 1024 * 1024;
        if (9ll * c * a.BN + 2 * stage + kSmemReserve + 8 * 1024 <= kSmemLimit) {
          a.rt_G = gg;
          break;
        }
      }
    }
    // rt_T * rt_G + 3 window rows: the right-border tap of the last output row reads index
    // (rows - 1) * P, the zero column of one more row (without it that read would reach the next
    // channel plane).
    a.rt_plane = (a.rt_T * a.rt_G + 3) * rt_P * 16;
    a.rt_box = a.rt_plane * (c / 16);
    // tap offsets read up to 2P + 2 pixels past a tile's 128 rows: slack after the last plane
    a.rt_stage = (a.rt_box + (2 * rt_P + 2 + 128) * 16 + 1023) / 1024 * 1024;
    CUtensorMap ma, mb;
    rc = encode_tiled_3d(&mb, d_w, static_cast<uint64_t>(9 * c), static_cast<uint64_t>(k), 1, a.BK, a.BN, a.BK);
    if (rc) return rc;
    rc = encode_rowtile(&ma, d_x, g.n, g.h, g.w, c, a.rt_P, a.rt_T * a.rt_G + 3);
    if (rc) return rc;
    g_last_path = 9;
    return launch_tc(*st, ma, mb, a, cs);
  }
  if (route.path == 15) {
    // G pixels per GEMM row: A = x as [M / G][G * C], B = block-diagonal weights in the stream's
    // workspace, output rows [G * K] = G NHWC pixels (residual likewise).
    const int G = route.group;
    const int kg = G * k, cg = G * c;
    const size_t wb = round256(static_cast<size_t>(kg) * cg), bb = round256(static_cast<size_t>(kg) * 4);
    void* ws = nullptr;
    rc = get_workspace(wb + 2 * bb, cs, &ws);
    if (rc) return rc;
    int8_t* wg = static_cast<int8_t*>(ws);
    int32_t* bg = reinterpret_cast<int32_t*>(static_cast<char*>(ws) + wb);
    float* sg = reinterpret_cast<float*>(static_cast<char*>(ws) + wb + bb);
    group_weights_kernel<<<grid_for(static_cast<size_t>(kg) * cg, 256, st->sms), 256, 0, cs>>>(
        d_w, wg, bg, sg, e.bias, e.scale, k, c, G);
    g_tc_launches.fetch_add(1, std::memory_order_relaxed);
    rc = check_launch("group_weights_kernel launch");
    if (rc) return rc;
    TcArgs a{};
    a.mode = 0;
    a.BK = route.tc_bk;
    a.cchunks = (cg + a.BK - 1) / a.BK;
    a.num_kb = a.cchunks;
    a.BN = pick_bn(kg, 0);
    a.M = static_cast<int>(M / G);
    a.N = kg;
    a.batch = 1;
    a.epi = e;
    if (e.bias) a.epi.bias = bg;
    if (e.scale) a.epi.scale = sg;
    a.out = d_y;
    a.ldc = kg;
    a.vec_ok = kg % 16 == 0;
    CUtensorMap ma, mb;
    rc = encode_tiled_3d(&ma, d_x, static_cast<uint64_t>(cg), static_cast<uint64_t>(a.M), 1, a.BK, kTcBM, a.BK);
    if (rc) return rc;
    rc = encode_tiled_3d(&mb, wg, static_cast<uint64_t>(cg), static_cast<uint64_t>(kg), 1, a.BK, a.BN, a.BK);
    if (rc) return rc;
    g_last_path = 15;
    return launch_tc(*st, ma, mb, a, cs);
  }
  if (route.path == 1 || route.path == 2 || route.path == 8) {
    TcArgs a{};
    a.BK = route.tc_bk;
    a.cchunks = (c + a.BK - 1) / a.BK;
    a.BN = pick_bn(k, 0);
    a.M = static_cast<int>(M);
    a.N = k;
    a.batch = 1;
    a.a_major = 0;
    a.b_major = 0;
    a.b_batched = 0;
    a.epi = e;
    a.out = d_y;
    a.ldc = k;
    a.batch_stride = 0;
    a.vec_ok = k % 16 == 0;
    a.conv_b = c % a.BK != 0;  // 3-D weight map only when the last K block needs zero fill
    CUtensorMap ma, mb;
    const int kdim = r * s * c;
    a.mode = is_1x1_plain ? 0 : 1;
    a.num_kb = is_1x1_plain ? a.cchunks : r * s * a.cchunks;
    a.pair = route.path == 8;
    if (a.conv_b)  // weights as {C, R*S, K}: a box of BK channels x 1 tap x BN output channels
      rc = encode_tiled_3d(&mb, d_w, static_cast<uint64_t>(c), static_cast<uint64_t>(r * s),
                           static_cast<uint64_t>(k), a.BK, 1, a.BK, a.BN);
    else  // weights as the K-major matrix [K][R*S*C] (half the N tile per box for 2-SM tiles)
      rc = encode_tiled_3d(&mb, d_w, static_cast<uint64_t>(kdim), static_cast<uint64_t>(k), 1, a.BK,
                           a.pair ? a.BN / 2 : a.BN, a.BK);
    if (rc) return rc;
    if (is_1x1_plain) {
      a.mode = 0;
      a.num_kb = a.cchunks;
      rc = encode_tiled_3d(&ma, d_x, static_cast<uint64_t>(c), static_cast<uint64_t>(M), 1, a.BK, kTcBM, a.BK);
      if (rc) return rc;
      g_last_path = a.pair ? 8 : 2;
    } else {
      a.mode = 1;
      a.num_kb = r * s * a.cchunks;
      a.Ho = g.ho; a.Wo = g.wo; a.S = s;
      a.stride_h = g.stride_h; a.stride_w = g.stride_w;
      a.pad_h = g.pad_h; a.pad_w = g.pad_w;
      a.dil_h = g.dil_h; a.dil_w = g.dil_w;
      rc = encode_im2col(&ma, d_x, g, a.BK);
      if (rc) return rc;
      g_last_path = 1;
    }
    // Long reductions consume operands faster than the TMA splits a B box into 128-byte row
    // requests: the weights go through one prepack pass into per-stage shared-memory images, then
    // one bulk copy per stage (one-CTA tiles, 128-byte K blocks, weights not resident).  The pass
    // costs a few microseconds, so only GEMMs of at least 2^36 MACs take it (config 4 layer 1:
    // 0.161-0.164 -> 0.155 ms; ResNet-50's 13-30 GMAC layers measured 1.5 % slower with it).
    const int n_tiles = (k + a.BN - 1) / a.BN;
    const bool b_res_like = n_tiles == 1 && static_cast<long long>(a.num_kb) * a.BN * a.BK <= 64 * 1024;
    const double macs = static_cast<double>(M) * k * a.num_kb * a.BK;
    if (g_b_prepack && !a.pair && a.BK == 128 && a.num_kb >= g_prepack_min_kb && !b_res_like && aligned16(d_w) &&
        macs >= 0x1p36) {
      const long long units = static_cast<long long>(n_tiles) * a.num_kb * a.BN * 8;
      void* ws = nullptr;
      rc = get_workspace(static_cast<size_t>(units) * 16, cs, &ws);
      if (rc) return rc;
      const int threads = 256;
      long long blocks = (units + threads - 1) / threads;
      if (blocks > 8 * st->sms) blocks = 8 * st->sms;
      pack_b_stages_kernel<<<static_cast<int>(blocks), threads, 0, cs>>>(d_w, static_cast<int8_t*>(ws), k, r * s, c,
                                                                         a.cchunks, a.num_kb, a.BN, units);
      g_tc_launches.fetch_add(1, std::memory_order_relaxed);
      rc = check_launch("pack_b_stages_kernel launch");
      if (rc) return rc;
      a.b_packed = static_cast<const int8_t*>(ws);
    }
    return launch_tc(*st, ma, mb, a, cs);
  }
  // Low-channel convolutions (C % 16 != 0): im2col pack into the stream's workspace, then tcgen05.
  // (tc_ok was false here, so a C % 16 == 0 conv reaching this point is one im2col TMA cannot take.)
  const int kp_packed = (r * s * c + 31) / 32 * 32;
  // Also taken by groups == 1 convs the im2col TMA cannot read (activations < 128 KiB, corner limits).
  if (route.path == 7) {
    void* ws = nullptr;
    rc = get_workspace(packed_scratch_bytes(M, k, kp_packed), cs, &ws);
    if (rc) return rc;
    g_last_path = 7;
    return run_packed_conv(*st, d_x, d_w, d_y, g, e, static_cast<int8_t*>(ws), cs);
  }
  if (route.path == 12) {
    DwPlan dp;
    dw_tma_plan(g, &dp);
    dp.wait_limit = wait_limit();
    dp.err = st->err;
    CUtensorMap mx;
    rc = encode_dw(&mx, d_x, g, dp);
    if (rc) return rc;
    const size_t smem = static_cast<size_t>(dp.stages) * dp.stage + 1024;
    int per_sm = static_cast<int>((kSmemLimit + 1024) / (smem + 1024));
    if (per_sm > 2) per_sm = 2;
    if (per_sm < 1) per_sm = 1;
    const int grid = dp.total < st->sms * per_sm ? dp.total : st->sms * per_sm;
    g_last_path = 12;
    const int cl = (e.zp == 0 && e.lo == -128 && e.hi == 127) ? 1 : (e.zp == 0 && e.lo == 0 && e.hi <= 127) ? 2 : 0;
    int8_t* yo = static_cast<int8_t*>(d_y);
#define B200Q_DW(S, CL) dw_tma_s8_kernel<S, CL><<<grid, kDwThreads, smem, cs>>>(mx, yo, d_w, g, e, dp)
    if (g.stride_h == 1) {
      if (cl == 1) B200Q_DW(1, 1); else if (cl == 2) B200Q_DW(1, 2); else B200Q_DW(1, 0);
    } else {
      if (cl == 1) B200Q_DW(2, 1); else if (cl == 2) B200Q_DW(2, 2); else B200Q_DW(2, 0);
    }
#undef B200Q_DW
    return check_launch("dw_tma_s8_kernel launch");
  }
  const size_t total = static_cast<size_t>(M) * k;
  if (route.path == 4) {
    const int groups8 = c / 8;
    const int lanes = 256 / groups8;
    g_last_path = 4;
    if (g_dw_px && g.dil_h == 1 && g.dil_w == 1 && (g.stride_w == 1 || g.stride_w == 2)) {
      // Several adjacent output pixels per thread share their input words.
      const int px = g.stride_w == 1 ? 8 : 2;
      const long long items = static_cast<long long>(g.n) * g.ho * ((g.wo + px - 1) / px);
      const long long blocks = (items + lanes - 1) / lanes;
      const int grid = static_cast<int>(blocks < st->sms * 8ll ? blocks : st->sms * 8ll);
      if (g.stride_w == 1) {
        if (e.out_kind == kOutS8)
          dw_conv_s8_px_kernel<kOutS8, 1, 8><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
        else if (e.out_kind == kOutS32)
          dw_conv_s8_px_kernel<kOutS32, 1, 8><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
        else
          dw_conv_s8_px_kernel<kOutF32, 1, 8><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
      } else {
        if (e.out_kind == kOutS8)
          dw_conv_s8_px_kernel<kOutS8, 2, 2><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
        else if (e.out_kind == kOutS32)
          dw_conv_s8_px_kernel<kOutS32, 2, 2><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
        else
          dw_conv_s8_px_kernel<kOutF32, 2, 2><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
      }
      return check_launch("dw_conv_s8_px_kernel launch");
    }
    const long long blocks = (M + lanes - 1) / lanes;
    const int grid = static_cast<int>(blocks < st->sms * 8ll ? blocks : st->sms * 8ll);
    if (e.out_kind == kOutS8)
      dw_conv_s8_kernel<kOutS8><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
    else if (e.out_kind == kOutS32)
      dw_conv_s8_kernel<kOutS32><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
    else
      dw_conv_s8_kernel<kOutF32><<<grid, 256, 0, cs>>>(d_x, d_w, d_y, g, e);
    g_last_path = 4;
    return check_launch("dw_conv_s8_kernel launch");
  }
  const int dp4a = (g.cg % 4 == 0) && (c % 4 == 0) && (reinterpret_cast<uintptr_t>(d_x) % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(d_w) % 4 == 0);
  conv_s8_generic_kernel<<<grid_for(total, 256, st->sms), 256, 0, cs>>>(d_x, d_w, d_y, g, e, dp4a);
  g_last_path = 3;
  return check_launch("conv_s8_generic_kernel launch");
}

int b200q_conv2d_s8_plan(int n, int h, int w, int c, int r, int s, int k, const b200q_conv_params* p,
                         const b200q_epilogue* epi, int has_residual, int* path) {
  if (!path) return fail(B200Q_ERR_INVALID_ARG, "null argument");
  ConvGeom g;
  int rc = conv_geom(n, h, w, c, r, s, k, p, 1, 1, &g);
  if (rc) return rc;
  if (!epi) return fail(B200Q_ERR_INVALID_ARG, "epilogue descriptor is null");
  if (epi->out_kind < 0 || epi->out_kind > 2) return fail(B200Q_ERR_INVALID_ARG, "bad out_kind %d", epi->out_kind);
  if (has_residual && epi->out_kind != B200Q_OUT_S8)
    return fail(B200Q_ERR_INVALID_ARG, "a residual add needs int8 outputs");
  int sms = 148;
  int dev = 0, count = 0;
  if (cudaGetDeviceCount(&count) == cudaSuccess && count > 0 && cudaGetDevice(&dev) == cudaSuccess) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
  } else {
    cudaGetLastError();  // no device here: clear the sticky error of the query
  }
  *path = route_conv_s8(g, h, w, c, r, s, k, true, true, true, true, has_residual != 0, epi->out_kind, sms).path;
  return B200Q_OK;
}

int b200q_conv2d_s8(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias, const float* d_scale, void* d_y,
                    int n, int h, int w, int c, int r, int s, int k, const b200q_conv_params* p,
                    const b200q_epilogue* epi, void* stream) {
  return conv2d_s8_impl(d_x, d_w, d_bias, d_scale, nullptr, 0.0f, d_y, n, h, w, c, r, s, k, p, epi, stream);
}

int b200q_conv2d_s8_add(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias, const float* d_scale,
                        const int8_t* d_res, float res_scale, int8_t* d_y, int n, int h, int w, int c, int r, int s,
                        int k, const b200q_conv_params* p, const b200q_epilogue* epi, void* stream) {
  if (!d_res) return fail(B200Q_ERR_INVALID_ARG, "residual pointer is null");
  return conv2d_s8_impl(d_x, d_w, d_bias, d_scale, d_res, res_scale, d_y, n, h, w, c, r, s, k, p, epi, stream);
}

int b200q_bmm_s8(const int8_t* A, const int8_t* B, const int32_t* d_bias, const float* d_col_scale, void* C,
                 int batch, int M, int N, int K, int trans_a, int trans_b, const b200q_epilogue* epi, void* stream) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(B200Q_ERR_INVALID_ARG, "negative bmm dimension");
  if (batch == 0 || M == 0 || N == 0) return B200Q_OK;
  if (!A || !B || !C) return fail(B200Q_ERR_INVALID_ARG, "null bmm pointer");
  Epilogue e{};
  int rc = make_epilogue(epi, d_bias, d_col_scale, &e);
  if (rc) return rc;
  DeviceState* st = nullptr;
  rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t cs = as_stream(stream);
  const bool ta = trans_a != 0, tb = trans_b != 0;
  const bool vec_ptrs = aligned16(A) && aligned16(B) && aligned16(C) && (!d_bias || aligned16(d_bias)) &&
                        (!d_col_scale || aligned16(d_col_scale));
  const bool tc_ok = g_policy.load() == 0 && K > 0 && vec_ptrs && (ta ? M % 16 == 0 : K % 16 == 0) &&
                     (tb ? K % 16 == 0 : N % 16 == 0);
  if (tc_ok) return bmm_s8_tcgen05(*st, A, B, C, batch, M, N, K, ta, tb, e, cs);
  {
    const long long tiles = static_cast<long long>((N + 63) / 64) * ((M + 63) / 64) * batch;
    const int blocks = static_cast<int>(tiles < 0x7fffffffll ? tiles : 0x7fffffffll);
    bmm_simt_kernel<int8_t><<<blocks, 256, 0, cs>>>(A, B, C, M, N, K, ta, tb, e, nullptr, 0, batch);
    rc = check_launch("bmm_simt_kernel<int8> launch");
    if (rc) return rc;
  }
  g_last_path = 3;
  return B200Q_OK;
}

int b200q_maxpool_s8(const int8_t* d_x, int8_t* d_y, int n, int h, int w, int c, int r, int s, int stride_h,
                     int stride_w, int pad_h, int pad_w, void* stream) {
  if (n < 0 || h <= 0 || w <= 0 || c <= 0 || r <= 0 || s <= 0) return fail(B200Q_ERR_INVALID_ARG, "bad pool shape");
  if (stride_h <= 0 || stride_w <= 0) return fail(B200Q_ERR_INVALID_ARG, "stride must be > 0");
  if (pad_h < 0 || pad_w < 0 || pad_h >= r || pad_w >= s)
    return fail(B200Q_ERR_INVALID_ARG, "padding must be >= 0 and smaller than the window");
  if (!d_x || !d_y) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  ConvGeom g{};
  g.n = n; g.h = h; g.w = w; g.c = c; g.r = r; g.s = s; g.k = c;
  g.ho = (h + 2 * pad_h - r) / stride_h + 1;
  g.wo = (w + 2 * pad_w - s) / stride_w + 1;
  g.pad_h = pad_h; g.pad_w = pad_w; g.stride_h = stride_h; g.stride_w = stride_w; g.dil_h = 1; g.dil_w = 1;
  g.groups = c; g.cg = 1; g.kg = 1; g.by = 1; g.bx = 1; g.bho = g.ho; g.bwo = g.wo;
  if (g.ho <= 0 || g.wo <= 0) return fail(B200Q_ERR_INVALID_ARG, "pool window larger than the padded input");
  if (n == 0) return B200Q_OK;
  if (c % 16 == 0 && !(aligned16(d_x) && aligned16(d_y)))
    return fail(B200Q_ERR_INVALID_ARG, "C %% 16 == 0 pools need 16-byte aligned tensors");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const size_t items = static_cast<size_t>(n) * g.ho * g.wo * (c % 16 == 0 ? c / 16 : c);
  maxpool_s8_kernel<<<grid_for(items, 256, st->sms), 256, 0, as_stream(stream)>>>(d_x, d_y, g);
  return check_launch("maxpool_s8_kernel launch");
}

int b200q_global_avgpool_s8(const int8_t* d_x, int8_t* d_y, int n, int h, int w, int c, void* stream) {
  if (n < 0 || h <= 0 || w <= 0 || c <= 0) return fail(B200Q_ERR_INVALID_ARG, "bad pool shape");
  if (static_cast<long long>(h) * w > (1 << 23)) return fail(B200Q_ERR_UNSUPPORTED, "pool window too large");
  if (!d_x || !d_y) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  if (n == 0) return B200Q_OK;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const size_t warps = static_cast<size_t>(n) * ((c + 31) / 32);
  global_avgpool_s8_kernel<<<grid_for(warps * 32, 256, st->sms), 256, 0, as_stream(stream)>>>(d_x, d_y, n, h * w, c);
  return check_launch("global_avgpool_s8_kernel launch");
}

// Packed low-channel conv with fixed scratch: see include/b200q.h.  Same arithmetic and kernels as
// the packed path of b200q_conv2d_s8, but the im2col matrix and padded weights go to the static
// array above instead of a workspace, and nothing is allocated.
int b200q_conv2d_s8_packed_noalloc(const int8_t* d_x, const int8_t* d_w, const int32_t* d_bias, const float* d_scale,
                                   void* d_y, int n, int h, int w, int c, int r, int s, int k,
                                   const b200q_conv_params* p, const b200q_epilogue* epi, void* stream) {
  ConvGeom g;
  int rc = conv_geom(n, h, w, c, r, s, k, p, 1, 1, &g);
  if (rc) return rc;
  if (!d_x || !d_w || !d_y) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  if (g.groups != 1) return fail(B200Q_ERR_UNSUPPORTED, "the fixed-scratch conv supports groups == 1 only");
  Epilogue e{};
  rc = make_epilogue(epi, d_bias, d_scale, &e);
  if (rc) return rc;
  if (!aligned16(d_y) || (d_bias && !aligned16(d_bias)) || (d_scale && !aligned16(d_scale)))
    return fail(B200Q_ERR_INVALID_ARG, "output, bias and scale must be 16-byte aligned");
  const long long rows = static_cast<long long>(n) * g.ho * g.wo;
  const int kp = (r * s * c + 31) / 32 * 32;
  if (kp > 16384) return fail(B200Q_ERR_UNSUPPORTED, "R*S*C = %d exceeds 16384", r * s * c);
  const size_t need = packed_scratch_bytes(rows, k, kp);
  if (rows >= (1ll << 31) || need > kNoAllocScratchBytes)
    return fail(B200Q_ERR_INVALID_ARG,
                "fixed-scratch conv needs %zu bytes of scratch (N*Ho*Wo*%d + K*%d, each rounded to 256) but the "
                "maximum is %zu; use b200q_conv2d_s8 or a smaller batch",
                need, kp, kp, kNoAllocScratchBytes);
  DeviceState* st = nullptr;
  rc = device_state(&st);
  if (rc) return rc;
  int8_t* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  g_last_path = 7;
  return run_packed_conv(*st, d_x, d_w, d_y, g, e, scratch, as_stream(stream));
}

size_t b200q_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int b200q_device_error(void) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, st->err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  if (v != 0) {
    const int zero = 0;
    cudaMemcpy(st->err, &zero, sizeof(int), cudaMemcpyHostToDevice);
    return fail(B200Q_ERR_TIMEOUT, "device wait ran out (code 0x%x)", v);
  }
  return B200Q_OK;
}

int b200q_selftest_wait_timeout(long long cycles) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  wait_timeout_probe_kernel<<<1, 32>>>(cycles > 0 ? cycles : 1000, st->err);
  rc = check_launch("wait_timeout_probe_kernel launch");
  if (rc) return rc;
  return b200q_device_error();
}

int b200q_fill_s8_uniform(int8_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id, int lo, int hi,
                          void* stream) {
  if (!d_out || lo > hi || lo < -128 || hi > 127) return fail(B200Q_ERR_INVALID_ARG, "bad fill arguments");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const uint64_t key = mix64(seed * 0x9E3779B97F4A7C15ull ^ mix64(tensor_id + 0x632BE59BD9B4E019ull));
  fill_s8_uniform_kernel<<<grid_for(count, 256, st->sms), 256, 0, as_stream(stream)>>>(
      d_out, count, key, lo, static_cast<uint64_t>(hi - lo + 1));
  return check_launch("fill_s8_uniform_kernel launch");
}

int b200q_fill_i32_uniform(int32_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id, int32_t lo, int32_t hi,
                           void* stream) {
  if (!d_out || lo > hi) return fail(B200Q_ERR_INVALID_ARG, "bad fill arguments");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const uint64_t key = mix64(seed * 0x9E3779B97F4A7C15ull ^ mix64(tensor_id + 0x632BE59BD9B4E019ull));
  fill_i32_uniform_kernel<<<grid_for(count, 256, st->sms), 256, 0, as_stream(stream)>>>(
      d_out, count, key, lo, static_cast<uint64_t>(static_cast<long long>(hi) - lo + 1));
  return check_launch("fill_i32_uniform_kernel launch");
}

int b200q_fill_s8_table(int8_t* d_out, size_t count, uint64_t seed, uint64_t tensor_id, const int8_t* d_table,
                        void* stream) {
  if (!d_out || !d_table) return fail(B200Q_ERR_INVALID_ARG, "bad fill arguments");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const uint64_t key = mix64(seed * 0x9E3779B97F4A7C15ull ^ mix64(tensor_id + 0x632BE59BD9B4E019ull));
  fill_s8_table_kernel<<<grid_for(count, 256, st->sms), 256, 0, as_stream(stream)>>>(d_out, count, key, d_table);
  return check_launch("fill_s8_table_kernel launch");
}

// Groups of a few channels (depthwise and the like) run on CUDA cores: a tensor-core GEMM per group
// would have 1-4 rows or columns (env B200Q_F32_DIRECT=0 keeps them on the GEMM route; the forced
// CUDA-core policy sends every fp32 conv here, for cross-checks).
static bool f32_use_direct(const ConvGeom& g) {
  static const bool on = [] {
    const char* v = getenv("B200Q_F32_DIRECT");
    return !(v && v[0] == '0');
  }();
  return g_policy.load() == 1 || (on && static_cast<long long>(g.cg) * g.kg <= 16);
}

static int f32_conv_common(const void* a, const void* b, const void* out, int n, int h, int w, int c, int r, int s,
                           int k, const b200q_conv_params* p, int by, int bx, ConvGeom* g, DeviceState** st) {
  int rc = conv_geom(n, h, w, c, r, s, k, p, by, bx, g);
  if (rc) return rc;
  if (!a || !b || !out) return fail(B200Q_ERR_INVALID_ARG, "null tensor pointer");
  if (!f32_sizes_ok(*g)) return fail(B200Q_ERR_UNSUPPORTED, "fp32 conv too large for one batched GEMM");
  return device_state(st);
}

int b200q_conv_fprop_f32(const float* d_x, const float* d_w, const float* d_bias, int bias_mode, float* d_y, int n,
                         int h, int w, int c, int r, int s, int k, const b200q_conv_params* p, int block_by,
                         int block_bx, void* stream) {
  ConvGeom g;
  DeviceState* st = nullptr;
  int rc = f32_conv_common(d_x, d_w, d_y, n, h, w, c, r, s, k, p, block_by, block_bx, &g, &st);
  if (rc) return rc;
  if (bias_mode != 0 && bias_mode != 1) return fail(B200Q_ERR_INVALID_ARG, "bad bias mode %d", bias_mode);
  if (f32_use_direct(g)) {
    const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
    f32_direct_fprop_kernel<<<grid_for(total, 256, st->sms), 256, 0, as_stream(stream)>>>(d_x, d_w, d_y, g, d_bias,
                                                                                        bias_mode);
    g_last_path = 14;
    return check_launch("f32_direct_fprop_kernel launch");
  }
  return f32_fprop(*st, d_x, d_w, d_bias, bias_mode, d_y, g, as_stream(stream));
}

int b200q_conv_bprop_f32(const float* d_dy, const float* d_w, float* d_dx, int n, int h, int w, int c, int r, int s,
                         int k, const b200q_conv_params* p, int block_by, int block_bx, void* stream) {
  ConvGeom g;
  DeviceState* st = nullptr;
  int rc = f32_conv_common(d_dy, d_w, d_dx, n, h, w, c, r, s, k, p, block_by, block_bx, &g, &st);
  if (rc) return rc;
  if (f32_use_direct(g)) {
    const size_t total = static_cast<size_t>(g.n) * g.h * g.w * g.c;
    f32_direct_bprop_kernel<<<grid_for(total, 256, st->sms), 256, 0, as_stream(stream)>>>(d_dy, d_w, d_dx, g);
    g_last_path = 14;
    return check_launch("f32_direct_bprop_kernel launch");
  }
  return f32_bprop(*st, d_dy, d_w, d_dx, g, as_stream(stream));
}

int b200q_conv_grad_f32(const float* d_x, const float* d_dy, float* d_dw, float* d_dbias, int bias_mode, int n, int h,
                        int w, int c, int r, int s, int k, const b200q_conv_params* p, int block_by, int block_bx,
                        void* stream) {
  ConvGeom g;
  DeviceState* st = nullptr;
  int rc = f32_conv_common(d_x, d_dy, d_dw, n, h, w, c, r, s, k, p, block_by, block_bx, &g, &st);
  if (rc) return rc;
  if (bias_mode != 0 && bias_mode != 1) return fail(B200Q_ERR_INVALID_ARG, "bad bias mode %d", bias_mode);
  if (f32_use_direct(g)) {
    cudaStream_t cs = as_stream(stream);
    const long long total = static_cast<long long>(g.k) * g.by * g.bx * g.r * g.s * g.cg;
    const int grid = static_cast<int>(total < st->sms * 16ll ? total : st->sms * 16ll);
    f32_direct_grad_kernel<<<grid, 256, 0, cs>>>(d_x, d_dy, d_dw, g);
    rc = check_launch("f32_direct_grad_kernel launch");
    if (rc) return rc;
    if (d_dbias) {
      const int entries = g.k * g.by * g.bx;
      f32_dbias_kernel<<<entries < st->sms * 8 ? entries : st->sms * 8, 256, 0, cs>>>(d_dy, d_dbias, g, bias_mode);
      rc = check_launch("f32_dbias_kernel launch");
      if (rc) return rc;
    }
    g_last_path = 14;
    return B200Q_OK;
  }
  return f32_grad(*st, d_x, d_dy, d_dw, d_dbias, bias_mode, g, as_stream(stream));
}

int b200q_bmm_f32(const float* A, const float* B, float* C, int batch, int M, int N, int K, int trans_a, int trans_b,
                  void* stream) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return fail(B200Q_ERR_INVALID_ARG, "negative bmm dimension");
  if (batch == 0 || M == 0 || N == 0) return B200Q_OK;
  if (!C || (K > 0 && (!A || !B))) return fail(B200Q_ERR_INVALID_ARG, "null bmm pointer");
  if (M >= (1 << 30) || N >= (1 << 30) || K >= (1 << 28) || batch >= (1 << 24))
    return fail(B200Q_ERR_UNSUPPORTED, "bmm too large");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t cs = as_stream(stream);
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(C, 0, static_cast<size_t>(batch) * M * N * sizeof(float), cs);
    return e == cudaSuccess ? B200Q_OK : cuda_fail(e, "cudaMemsetAsync(bmm C)");
  }
  F32Pack qa{}, qb{};
  qa.mode = qb.mode = kPackMat;
  qa.rows = M; qb.rows = N;
  qa.cols = qb.cols = K;
  qa.kp = qb.kp = (K + 31) / 32 * 32;
  qa.lo_mask = 4; qb.lo_mask = 2;
  qa.batch = qb.batch = batch;
  // A [b][M][K] (or [b][K][M] transposed), B [b][K][N] (or [b][N][K] transposed): logical rows are
  // the output rows / columns, logical columns the reduction
  qa.sb = static_cast<long long>(M) * K;
  qa.sr = trans_a ? 1 : K;
  qa.sc = trans_a ? M : 1;
  qb.sb = static_cast<long long>(K) * N;
  qb.sr = trans_b ? K : 1;
  qb.sc = trans_b ? 1 : N;
  const size_t a_bytes = round256(static_cast<size_t>(batch) * M * 3 * qa.kp * 4);
  const size_t b_bytes = round256(static_cast<size_t>(batch) * N * 3 * qb.kp * 4);
  void* ws = nullptr;
  rc = get_workspace(a_bytes + b_bytes, cs, &ws);
  if (rc) return rc;
  float* ap = static_cast<float*>(ws);
  float* bp = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + a_bytes);
  if ((rc = f32_pack(*st, A, ap, qa, cs))) return rc;
  if ((rc = f32_pack(*st, B, bp, qb, cs))) return rc;
  if ((rc = f32_gemm(*st, ap, bp, C, batch, M, N, qa.kp, N, static_cast<long long>(M) * N, cs))) return rc;
  g_last_path = 13;
  return B200Q_OK;
}

}  // extern "C"
