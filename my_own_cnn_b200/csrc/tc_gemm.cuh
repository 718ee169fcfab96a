// Persistent, warp-specialised tcgen05 int8 GEMM engine for sm_100a.
//
// One CTA per SM, 320 threads:
//   warp 0      TMA producer (one elected lane): A tile (tiled 3-D map, or im2col 4-D map for
//               convolutions) and B tile into a `stages`-deep shared-memory ring;
//   warp 1      owns TMEM (alloc/dealloc) and issues tcgen05.mma.kind::i8 from one lane;
//               accumulators are double-buffered in TMEM (2 x BN columns of int32);
//   warps 2..9  epilogue: tcgen05.ld of the accumulator rows (warp w reads TMEM lanes
//               32*(w%4)..+31; two warps per lane quarter take alternating 32-column chunks),
//               fused bias / scale / round / clamp / pack, 16-byte stores.
// The GEMM is C[b][m][n] = sum_k A[b][m][k] * B[b][n][k] with M tile 128, N tile BN, K block BK
// bytes (= int8 elements).  For a convolution, m = (image, ho, wo), n = output channel,
// k = (r, s, c) -- the im2col TMA gathers the activation rows directly from NHWC memory, with
// zero fill for padding, so no im2col matrix is ever written.
//
// Every mbarrier wait is bounded (clock64 limit); on expiry a role records an error code in the
// device error word and leaves its loop; the CTA then drains its MMAs and frees TMEM.
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace b200q {

#ifndef B200Q_EPI_PER_QUARTER
#define B200Q_EPI_PER_QUARTER 2
#endif
constexpr int kTcEpiPerQuarter = B200Q_EPI_PER_QUARTER;  // epilogue warps per TMEM lane quarter
constexpr int kTcEpiWarps = 4 * kTcEpiPerQuarter;
constexpr int kTcThreads = 64 + 32 * kTcEpiWarps;  // producer warp, MMA warp, epilogue warps
constexpr int kTcBM = 128;

struct TcArgs {
  int mode;  // 0 = tiled 3-D A map, 1 = im2col A map
  int M, N;  // GEMM rows / cols per batch item
  int batch;
  int BN, BK, stages, num_kb;
  int m_tiles, n_tiles, total_tiles;
  int a_major, b_major;  // 0 = K-major, 1 = MN-major (bmm transposes)
  int b_batched;         // B map has a batch dimension (bmm); conv weights are shared
  int conv_b;            // B is conv weights as a 3-D map {C, R*S, K}: channels past C read as zero
  // im2col geometry
  int Ho, Wo, S, cchunks, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
  // epilogue
  Epilogue epi;
  void* out;
  long long ldc;            // elements between output rows
  long long batch_stride;   // elements between output batch items
  int vec_ok;               // rows and bias/scale allow 16-byte vector stores
  int vec8_ok;              // int8 rows allow 8-byte vector stores (N % 8 == 0; bias / scale staged)
  uint32_t idesc;
  uint32_t tmem_cols;
  int nacc;           // TMEM accumulator buffers (nacc x BN columns), 2..kTcMaxAcc
  long long wait_limit;
  int* err;
  int stage_cols;     // bias/scale columns copied to shared memory at start (0 = read from global)
  int default_clamp;  // int8 output with zp 0 and bounds [-128, 127]: saturating pack does the clamp
  int tma_store;      // outputs leave through shared memory + TMA tensor stores (map tmC)
  int b_res;          // B resident: all num_kb K blocks of the single N tile loaded once per CTA
  int pair;           // 2-SM tiles (tc_gemm_s8_pair_kernel): 256-row tiles, B box of BN / 2 rows
  // mode 2 (row tiles, 3x3 stride-1 convs): a tile is rt_T output rows of one image at row pitch
  // rt_P = Wo + 1; its input window (rt_T + 3 rows x rt_P columns x C, column 0 the zero padding)
  // arrives as one TMA box laid out [C / 16][pixel][16 B] (plane stride rt_plane bytes) and serves
  // all nine taps.
  int rt_P, rt_T, rt_plane;
  int rt_box;    // bytes of one window box (rt_plane * C / 16)
  int n_img;     // images (row tiles enumerate image x block of output rows)
  int rt_stage;  // ring stage size for row tiles (window + read-past slack, 1024-aligned)
  int rt_x0, rt_y0;  // window origin relative to (output column 0, the tile's first output row)
  // Tap-pair row tiles (space-to-depth stems): 16 channels per pixel, rt_R x rt_S taps, and each
  // K = 32 MMA slice covers taps (r, s) and (r, s + 1): the A descriptor's K-direction core
  // matrix stride is one pixel (rt_plane = 16), so the second half of the slice is the next pixel.
  int rt_pairs, rt_R, rt_S;
  int rt_wide;  // window map in 8-byte elements {2 * W, H, N} (one channel plane): rows of whole pixels
  // Row groups (tap-pair row tiles): a tile is rt_G groups of rt_T output rows sharing one window;
  // group j accumulates into TMEM columns [j * BN, (j + 1) * BN) of the buffer, from the window
  // started j * rt_T rows lower.  acc_cols = BN * rt_G columns per accumulator buffer.
  int rt_G, acc_cols;
  float hi_f;   // float(epi.hi), for the float-domain clamp of quant4_s8<2>
  int ab_unsigned;  // both operands unsigned 8-bit (the quantized-int32 drop-in's U8 codes)
  int tf32;         // fp32 operands, kind::tf32 MMAs, fp32 accumulators copied out bit for bit
  int kb_third;     // fp32 im2col convs: K blocks per third of the split reduction (0 otherwise)
  int grp_bytes;    // fp32 im2col convs: bytes between the channel starts of consecutive groups (batch items)
  // int8 TMA stores of 32 rows x 128 columns: each epilogue warp takes 4 adjacent chunks of a
  // 256-column tile and stores them with one 128-byte-wide box (SWIZZLE_128B map) instead of four
  // 32-byte-wide ones (requires BN = 256, N % 256 == 0, two warps per lane quarter).
  int wide_store;
  // Prepacked B (conv weights, 128-byte K blocks): stage image of (N tile nt, K block kb) at
  // b_packed + (nt * num_kb + kb) * BN * 128, exactly the shared-memory bytes the tensor-map load
  // would write (SWIZZLE_128B rows).  One bulk copy per stage instead of BN row requests.
  const int8_t* b_packed;
};

constexpr int kTcMaxAcc = 8;
constexpr int kEpiStageBytes = 32 * 128;   // one warp's 32 rows x 32 four-byte columns
constexpr int kEpiStageBytesS8 = 32 * 32;  // one warp's 32 rows x 32 int8 columns
constexpr int kEpiStageBytesS8W = 32 * 128;  // wide stores: 32 rows x 128 int8 columns

__device__ __forceinline__ uint32_t kmajor_layout(int bk) {
  return bk == 128 ? 2u : (bk == 64 ? 4u : 6u);  // SWIZZLE_128B / 64B / 32B
}

// Pack the low bytes of four ints into one word (byte i = value i).
__device__ __forceinline__ uint32_t pack4_s8(int a, int b, int c, int d) {
  const uint32_t lo = __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x0040);
  const uint32_t hi = __byte_perm(static_cast<uint32_t>(c), static_cast<uint32_t>(d), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}
// Pack four int32 into int8 bytes (byte i = value i) with saturation to [-128, 127].
__device__ __forceinline__ uint32_t pack4_sat_s8(int a, int b, int c, int d) {
  uint32_t out;
  asm("{\n\t.reg .b32 hi;\n\t"
      "cvt.pack.sat.s8.s32.b32 hi, %4, %3, 0;\n\t"
      "cvt.pack.sat.s8.s32.b32 %0, %2, %1, hi;\n\t}"
      : "=r"(out)
      : "r"(a), "r"(b), "r"(c), "r"(d));
  return out;
}

// Four requantized int8 codes packed in a word: clamp(rint_sat(f), lo - zp, hi - zp) + zp.
// CL selects how the clamp is done: 0 in integers (any bounds and zero point); 1 by the
// saturating pack alone (the default range [-128, 127], zero point 0); 2 in floats before the
// conversion (zero point 0 and lo = 0, the ReLU / ReLU6 forms: max(NaN, 0) = 0 matches
// rint_sat(NaN) = 0, and integer bounds commute with rounding), the upper bound 127 by the pack;
// 4 as 2 when hi >= 127 (plain ReLU): only the lower bound in floats, the pack does the rest.
template <int CL>
__device__ __forceinline__ uint32_t quant4_s8(const TcArgs& a, float f0, float f1, float f2, float f3) {
  const Epilogue& e = a.epi;
  if constexpr (CL == 2) {
    const float hi = a.hi_f;
    f0 = fminf(fmaxf(f0, 0.0f), hi); f1 = fminf(fmaxf(f1, 0.0f), hi);
    f2 = fminf(fmaxf(f2, 0.0f), hi); f3 = fminf(fmaxf(f3, 0.0f), hi);
  }
  if constexpr (CL == 4) {  // ReLU with upper bound >= 127: the saturating pack is the upper clamp
    f0 = fmaxf(f0, 0.0f); f1 = fmaxf(f1, 0.0f); f2 = fmaxf(f2, 0.0f); f3 = fmaxf(f3, 0.0f);
  }
  int r0 = __float2int_rn(f0), r1 = __float2int_rn(f1), r2 = __float2int_rn(f2), r3 = __float2int_rn(f3);
  if constexpr (CL == 0) {
    const int lo = e.lo - e.zp, hi = e.hi - e.zp;
    r0 = min(max(r0, lo), hi) + e.zp; r1 = min(max(r1, lo), hi) + e.zp;
    r2 = min(max(r2, lo), hi) + e.zp; r3 = min(max(r3, lo), hi) + e.zp;
  }
  return pack4_sat_s8(r0, r1, r2, r3);
}

// Coordinates (b, mt, nt) of tile index b * (m_tiles * n_tiles) + mt * n_tiles + nt, advanced
// by a fixed stride with carries (the persistent loops visit tile, tile + stride, ...).
struct TileWalk {
  int b, mt, nt;
  int m_tiles, n_tiles, inc_b, inc_mt, inc_nt;
  __device__ __forceinline__ TileWalk(int tile, int stride, int batch, int m_tiles_, int n_tiles_)
      : m_tiles(m_tiles_), n_tiles(n_tiles_) {
    const int per_b = m_tiles * n_tiles;
    b = tile / per_b;
    const int rem = tile - b * per_b;
    mt = rem / n_tiles;
    nt = rem - mt * n_tiles;
    inc_b = stride / per_b;
    const int srem = stride - inc_b * per_b;
    inc_mt = srem / n_tiles;
    inc_nt = srem - inc_mt * n_tiles;
    (void)batch;
  }
  __device__ __forceinline__ void next() {
    nt += inc_nt;
    int c = 0;
    if (nt >= n_tiles) {
      nt -= n_tiles;
      c = 1;
    }
    mt += inc_mt + c;
    b += inc_b;
    if (mt >= m_tiles) {
      mt -= m_tiles;
      ++b;
    }
  }
};

// Vector form of the fused epilogue: the first 4 * NQ columns of the chunk (NQ = 8: all 32,
// NQ = 4: the first 16), 16-byte bias / scale reads and 16-byte stores.
template <int KIND, int CL, int NQ, bool RES>
__device__ __forceinline__ void store_vec(const TcArgs& a, const uint32_t (&v)[32], size_t off, int n,
                                          const int32_t* bias, const float* scale, bool has_bias) {
  const Epilogue& e = a.epi;
  const int4* bp = reinterpret_cast<const int4*>(bias + n);
  const float4* sp = reinterpret_cast<const float4*>(scale + n);
  uint32_t packed[8];
  uint32_t rw[8];  // residual bytes of this row's columns (RES only)
  if constexpr (RES) {
    const uint4 r0 = *reinterpret_cast<const uint4*>(e.res + off);
    rw[0] = r0.x; rw[1] = r0.y; rw[2] = r0.z; rw[3] = r0.w;
    if constexpr (NQ == 8) {
      const uint4 r1 = *reinterpret_cast<const uint4*>(e.res + off + 16);
      rw[4] = r1.x; rw[5] = r1.y; rw[6] = r1.z; rw[7] = r1.w;
    }
  }
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    int t0 = static_cast<int>(v[4 * q + 0]), t1 = static_cast<int>(v[4 * q + 1]);
    int t2 = static_cast<int>(v[4 * q + 2]), t3 = static_cast<int>(v[4 * q + 3]);
    if (has_bias) {
      const int4 bb = bp[q];
      t0 = wrap_add(t0, bb.x); t1 = wrap_add(t1, bb.y); t2 = wrap_add(t2, bb.z); t3 = wrap_add(t3, bb.w);
    }
    if constexpr (KIND == kOutS32) {
      reinterpret_cast<int4*>(static_cast<int32_t*>(a.out) + off)[q] = make_int4(t0, t1, t2, t3);
    } else {
      const float4 s4 = sp[q];
      const float p0 = __fmul_rn(__int2float_rn(t0), s4.x), p1 = __fmul_rn(__int2float_rn(t1), s4.y);
      const float p2 = __fmul_rn(__int2float_rn(t2), s4.z), p3 = __fmul_rn(__int2float_rn(t3), s4.w);
      if constexpr (KIND == kOutF32) {
        reinterpret_cast<float4*>(static_cast<float*>(a.out) + off)[q] = make_float4(p0, p1, p2, p3);
      } else {
        float f0 = p0, f1 = p1, f2 = p2, f3 = p3;
        if constexpr (RES) {
          f0 = __fadd_rn(f0, __fmul_rn(__int2float_rn(sbyte(rw[q], 0)), e.res_scale));
          f1 = __fadd_rn(f1, __fmul_rn(__int2float_rn(sbyte(rw[q], 1)), e.res_scale));
          f2 = __fadd_rn(f2, __fmul_rn(__int2float_rn(sbyte(rw[q], 2)), e.res_scale));
          f3 = __fadd_rn(f3, __fmul_rn(__int2float_rn(sbyte(rw[q], 3)), e.res_scale));
        }
        packed[q] = quant4_s8<CL>(a, f0, f1, f2, f3);
      }
    }
  }
  if constexpr (KIND == kOutS8) {
    int4* o = reinterpret_cast<int4*>(static_cast<int8_t*>(a.out) + off);
    o[0] = make_int4(packed[0], packed[1], packed[2], packed[3]);
    if constexpr (NQ == 8) o[1] = make_int4(packed[4], packed[5], packed[6], packed[7]);
  }
}

// int8 output of the first 4 * NQ columns of a chunk (NQ even) with 8-byte residual loads and
// stores: rows of N % 16 == 8 bytes (N = 24, 40, ...) are only 8-byte aligned.  The arithmetic is
// store_vec's.
template <int CL, int NQ, bool RES>
__device__ __forceinline__ void store_vec8(const TcArgs& a, const uint32_t (&v)[32], size_t off, int n,
                                           const int32_t* bias, const float* scale, bool has_bias) {
  const Epilogue& e = a.epi;
  const int4* bp = reinterpret_cast<const int4*>(bias + n);
  const float4* sp = reinterpret_cast<const float4*>(scale + n);
  uint32_t packed[NQ];
  uint32_t rw[NQ];
  if constexpr (RES) {
#pragma unroll
    for (int i = 0; i < NQ / 2; ++i) {
      const uint2 r = *reinterpret_cast<const uint2*>(e.res + off + 8 * i);
      rw[2 * i] = r.x;
      rw[2 * i + 1] = r.y;
    }
  }
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    int t0 = static_cast<int>(v[4 * q + 0]), t1 = static_cast<int>(v[4 * q + 1]);
    int t2 = static_cast<int>(v[4 * q + 2]), t3 = static_cast<int>(v[4 * q + 3]);
    if (has_bias) {
      const int4 bb = bp[q];
      t0 = wrap_add(t0, bb.x); t1 = wrap_add(t1, bb.y); t2 = wrap_add(t2, bb.z); t3 = wrap_add(t3, bb.w);
    }
    const float4 s4 = sp[q];
    float f0 = __fmul_rn(__int2float_rn(t0), s4.x), f1 = __fmul_rn(__int2float_rn(t1), s4.y);
    float f2 = __fmul_rn(__int2float_rn(t2), s4.z), f3 = __fmul_rn(__int2float_rn(t3), s4.w);
    if constexpr (RES) {
      f0 = __fadd_rn(f0, __fmul_rn(__int2float_rn(sbyte(rw[q], 0)), e.res_scale));
      f1 = __fadd_rn(f1, __fmul_rn(__int2float_rn(sbyte(rw[q], 1)), e.res_scale));
      f2 = __fadd_rn(f2, __fmul_rn(__int2float_rn(sbyte(rw[q], 2)), e.res_scale));
      f3 = __fadd_rn(f3, __fmul_rn(__int2float_rn(sbyte(rw[q], 3)), e.res_scale));
    }
    packed[q] = quant4_s8<CL>(a, f0, f1, f2, f3);
  }
  uint2* o = reinterpret_cast<uint2*>(static_cast<int8_t*>(a.out) + off);
#pragma unroll
  for (int i = 0; i < NQ / 2; ++i) o[i] = make_uint2(packed[2 * i], packed[2 * i + 1]);
}

// Fused epilogue for one row and 32 consecutive output columns [n, n + valid).
// bias / scale point at shared memory (staged) or global memory; bias may be null.
// All array indices are compile-time constants after unrolling: nothing spills to local memory.
template <int KIND, int CL, bool RES>
__device__ __forceinline__ void store_chunk(const TcArgs& a, const uint32_t (&v)[32], size_t off, int n, int valid,
                                            const int32_t* bias, const float* scale, bool has_bias) {
  const Epilogue& e = a.epi;
  if constexpr (KIND == kOutS8) {
    if (!a.vec_ok && a.vec8_ok) {  // N % 16 == 8: 8-byte rows
      if (valid == 32) {
        store_vec8<CL, 8, RES>(a, v, off, n, bias, scale, has_bias);
        return;
      }
      if (valid == 24) {
        store_vec8<CL, 6, RES>(a, v, off, n, bias, scale, has_bias);
        return;
      }
      if (valid == 8) {
        store_vec8<CL, 2, RES>(a, v, off, n, bias, scale, has_bias);
        return;
      }
    }
  }
  if (a.vec_ok) {
    if (valid == 32) {
      store_vec<KIND, CL, 8, RES>(a, v, off, n, bias, scale, has_bias);
      return;
    }
    if (valid == 16) {  // the 16-column tail of N = 16, 48, 80, ...
      store_vec<KIND, CL, 4, RES>(a, v, off, n, bias, scale, has_bias);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < valid) {
      int t = static_cast<int>(v[j]);
      if (has_bias) t = wrap_add(t, bias[n + j]);
      if constexpr (KIND == kOutS32) {
        static_cast<int32_t*>(a.out)[off + j] = t;
      } else if constexpr (KIND == kOutF32) {
        static_cast<float*>(a.out)[off + j] = __fmul_rn(__int2float_rn(t), scale[n + j]);
      } else if constexpr (RES) {
        static_cast<int8_t*>(a.out)[off + j] =
            static_cast<int8_t>(requant_res(t, scale[n + j], e.res[off + j], e.res_scale, e));
      } else {
        static_cast<int8_t*>(a.out)[off + j] = static_cast<int8_t>(requant_one(t, scale[n + j], e));
      }
    }
  }
}

// 4-byte outputs through shared memory: the warp's 32x32 block is written into a 128B-swizzled
// buffer (16-byte chunk j of row r at chunk j ^ (r % 8), the layout of a SWIZZLE_128B tensor map)
// and stored by one TMA instruction, which also clips rows >= M and columns >= N.
template <int KIND>
__device__ __forceinline__ void stage_chunk_4b(const TcArgs& a, const uint32_t (&v)[32], int n, int lane,
                                               uint8_t* sbuf, const int32_t* bias, const float* scale,
                                               bool has_bias) {
  const bool full = n + 32 <= a.N;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    int t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int col = n + 4 * q + i;
      t[i] = static_cast<int>(v[4 * q + i]);
      if (has_bias && (full || col < a.N)) t[i] = wrap_add(t[i], bias[col]);
    }
    uint4 w;
    if constexpr (KIND == kOutS32) {
      w = make_uint4(t[0], t[1], t[2], t[3]);
    } else {
      float f[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = n + 4 * q + i;
        f[i] = (full || col < a.N) ? __fmul_rn(__int2float_rn(t[i]), scale[col]) : 0.0f;
      }
      w = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    *reinterpret_cast<uint4*>(sbuf + lane * 128 + ((q ^ (lane & 7)) << 4)) = w;
  }
}

// int8 outputs through shared memory: the warp's 32 rows x 32 bytes are written into a
// 32B-swizzled 1 KiB buffer (16-byte half h of row r at half h ^ ((r / 4) % 2), the layout of a
// SWIZZLE_32B tensor map: conflict-free for one 16-byte store per lane) and leave with one TMA
// store, which clips rows >= M and columns >= N.  The requantization is the one of store_chunk.
template <int CL, bool RES, bool WIDE>
__device__ __forceinline__ void stage_chunk_s8(const TcArgs& a, const uint32_t (&v)[32], int n, int lane,
                                               uint8_t* sbuf, const int32_t* bias, const float* scale,
                                               bool has_bias, const int8_t* rrow, int slot) {
  const Epilogue& e = a.epi;
  const int4* bp = reinterpret_cast<const int4*>(bias + n);
  const float4* sp = reinterpret_cast<const float4*>(scale + n);
  uint32_t packed[8];
  uint32_t rw[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // residual bytes of the row (RES; rows past M read none)
  if constexpr (RES) {
    if (rrow) {
      const bool full = n + 32 <= a.N;
      const uint4 r0 = *reinterpret_cast<const uint4*>(rrow);
      rw[0] = r0.x; rw[1] = r0.y; rw[2] = r0.z; rw[3] = r0.w;
      if (full || n + 16 < a.N) {
        const uint4 r1 = *reinterpret_cast<const uint4*>(rrow + 16);
        rw[4] = r1.x; rw[5] = r1.y; rw[6] = r1.z; rw[7] = r1.w;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    int t0 = static_cast<int>(v[4 * q + 0]), t1 = static_cast<int>(v[4 * q + 1]);
    int t2 = static_cast<int>(v[4 * q + 2]), t3 = static_cast<int>(v[4 * q + 3]);
    if (has_bias) {
      const int4 bb = bp[q];
      t0 = wrap_add(t0, bb.x); t1 = wrap_add(t1, bb.y); t2 = wrap_add(t2, bb.z); t3 = wrap_add(t3, bb.w);
    }
    const float4 s4 = sp[q];
    float f0 = __fmul_rn(__int2float_rn(t0), s4.x), f1 = __fmul_rn(__int2float_rn(t1), s4.y);
    float f2 = __fmul_rn(__int2float_rn(t2), s4.z), f3 = __fmul_rn(__int2float_rn(t3), s4.w);
    if constexpr (RES) {
      f0 = __fadd_rn(f0, __fmul_rn(__int2float_rn(sbyte(rw[q], 0)), e.res_scale));
      f1 = __fadd_rn(f1, __fmul_rn(__int2float_rn(sbyte(rw[q], 1)), e.res_scale));
      f2 = __fadd_rn(f2, __fmul_rn(__int2float_rn(sbyte(rw[q], 2)), e.res_scale));
      f3 = __fadd_rn(f3, __fmul_rn(__int2float_rn(sbyte(rw[q], 3)), e.res_scale));
    }
    packed[q] = quant4_s8<CL>(a, f0, f1, f2, f3);
  }
  if constexpr (WIDE) {
    // 128-byte rows, SWIZZLE_128B: 16-byte unit j of row r at unit j ^ (r % 8); this chunk is
    // units 2 * slot and 2 * slot + 1 of the row.
    const int x = lane & 7;
    *reinterpret_cast<uint4*>(sbuf + lane * 128 + (((2 * slot) ^ x) << 4)) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
    *reinterpret_cast<uint4*>(sbuf + lane * 128 + (((2 * slot + 1) ^ x) << 4)) =
        make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else {
    (void)slot;
    const int sw = (lane >> 2) & 1;
    *reinterpret_cast<uint4*>(sbuf + lane * 32 + (sw << 4)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    *reinterpret_cast<uint4*>(sbuf + lane * 32 + ((sw ^ 1) << 4)) =
        make_uint4(packed[4], packed[5], packed[6], packed[7]);
  }
}

// Epilogue role: 8 warps; warp w reads TMEM lanes 32*(w%4)..+31 (the hardware restricts a warp
// to the lane quarter w%4) and, in the j-th tile of its CTA, the chunks of 32 columns with
// chunk % 2 == ((w-2)/4 + j) % 2.  Each chunk is loaded and processed in turn: overlapping the
// next chunk's TMEM load with two register buffers measured slower (the extra register moves
// cost more issue slots than the load latency it hid).
template <int KIND, bool TMA, int CL, bool RES, bool WIDE>
__device__ __forceinline__ void emit_chunk(const TcArgs& a, const CUtensorMap* tmC, const uint32_t (&v)[32], int b,
                                           int m, int mrow0, size_t row_off, int n, int lane, uint8_t* sbufs,
                                           int& sb, const int32_t* bias, const float* scale,
                                           bool has_bias, int slot, bool last) {
  if constexpr (WIDE) {
    // slot 0..3 of this warp's 128-column block; the box leaves after the warp's last valid chunk
    // (the TMA store clips columns >= N, so unwritten slots past N never reach memory)
    uint8_t* buf = sbufs + sb * kEpiStageBytesS8W;
    if (slot == 0) {
      if (lane == 0) bulk_wait_group_read<1>();  // the store that used this buffer has read it
      __syncwarp();
    }
    stage_chunk_s8<CL, RES, true>(a, v, n, lane, buf, bias, scale, has_bias,
                                  RES && m < a.M ? a.epi.res + row_off + n : nullptr, slot);
    if (last) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(tmC, smem_u32(buf), n - 32 * slot, mrow0, b);
        bulk_commit_group();
      }
      sb ^= 1;
    }
    return;
  }
  if (n >= a.N) return;
  if constexpr (TMA) {
    uint8_t* buf = sbufs + sb * (KIND == kOutS8 ? kEpiStageBytesS8 : kEpiStageBytes);
    if (lane == 0) bulk_wait_group_read<1>();  // the store that used this buffer has read it
    __syncwarp();
    if constexpr (KIND == kOutS8)
      stage_chunk_s8<CL, RES, false>(a, v, n, lane, buf, bias, scale, has_bias,
                                      RES && m < a.M ? a.epi.res + row_off + n : nullptr, -1);
    else
      stage_chunk_4b<KIND>(a, v, n, lane, buf, bias, scale, has_bias);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmC, smem_u32(buf), n, mrow0, b);
      bulk_commit_group();
    }
    sb ^= 1;
    return;
  }
  if (m < a.M) store_chunk<KIND, CL, RES>(a, v, row_off + n, n, min(32, a.N - n), bias, scale, has_bias);
}

// PAIR: the CTA is one half of a 2-SM pair (tiles of 2 x 128 rows; this CTA's TMEM holds rows
// rank * 128 .. + 127 of each tile; the accumulator-empty barrier lives in the leader CTA).
template <int KIND, bool TMA, int CL, bool PAIR, bool RES, bool WIDE>
__device__ __forceinline__ void epilogue_role_t(const TcArgs& a, const CUtensorMap* tmC, uint32_t tmem_base,
                                              uint32_t accf0, uint32_t acce0, int warp, int lane,
                                              const int32_t* bias, const float* scale, bool has_bias,
                                              uint8_t* sbufs) {
  int sb = 0;
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int rank = PAIR ? static_cast<int>(cluster_ctarank()) : 0;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nunits = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  constexpr int TM = PAIR ? 2 * kTcBM : kTcBM;
  const int row = rank * kTcBM + q * 32 + lane;
  int buf = 0;
  uint32_t acc_ph = 0;
  int sel = half;  // this warp's chunks in the current tile: sel, sel + E, ... (E warps per quarter)
  // Tile coordinates advance by `nunits` tiles per iteration as mixed-radix counters (batch item,
  // M tile, N tile; for row tiles image and block of output rows): no integer division per tile.
  TileWalk tw(unit, nunits, a.batch, a.m_tiles, a.n_tiles);
  const bool rt = !PAIR && a.mode == 2;
  const int rt_tb = a.rt_T * a.rt_G;  // output rows per tile
  const int rblocks = rt ? (a.Ho + rt_tb - 1) / rt_tb : 1;
  TileWalk rw(rt ? unit : 0, nunits, 1 << 30, rblocks, 1);  // (image, row block) of mode-2 tiles
  // Row tile: TMEM row -> (tile row ti, column wo) at pitch P; pitch padding and rows past the
  // tile or the image are not stored.
  const int ti = rt ? row / a.rt_P : 0, two = rt ? row - ti * a.rt_P : 0;
  for (int tile = unit; tile < a.total_tiles;
       tile += nunits, sel = (sel + 1 == kTcEpiPerQuarter ? 0 : sel + 1), tw.next(), rw.next()) {
    const int b = tw.b, mt = tw.mt, nt = tw.nt;
    int m = mt * TM + row;
    const int n0 = nt * a.BN;
    size_t rt_off = 0;
    int rt_img = 0, rt_ho0 = 0;
    if (rt) {
      rt_img = rw.b;
      rt_ho0 = rw.mt * rt_tb;
      const bool valid = ti < a.rt_T && rt_ho0 + ti < a.Ho && two < a.Wo;
      m = valid ? 0 : a.M;
      rt_off = (static_cast<size_t>(rt_img * a.Ho + rt_ho0 + ti) * a.Wo + two) * a.ldc;
    }
    // Chunks holding columns < N (times the row groups); the warps of a lane quarter rotate through
    // them every tile, so an odd chunk count (N <= 32, N = 96, ...) is shared evenly over tiles.
    const int ncols = (min(a.BN, a.N - n0) + 31) >> 5;
    const int nvalid = ncols * a.rt_G;
    const int nmine = WIDE ? max(0, min(4, nvalid - 4 * sel))
                           : (nvalid > sel ? (nvalid - sel + kTcEpiPerQuarter - 1) / kTcEpiPerQuarter : 0);
    if (!mbar_wait_bounded(accf0 + 8 * buf, acc_ph, a.wait_limit, a.err, kDevErrTimeoutEpilogue)) break;
    tc_fence_after();
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * a.acc_cols);
    const size_t row_off =
        (!PAIR && a.mode == 2) ? rt_off : static_cast<size_t>(b) * a.batch_stride + static_cast<size_t>(m) * a.ldc;
    const int mrow0 = mt * TM + rank * kTcBM + q * 32;
    // int32 outputs with per-row terms: t = acc + rowterm[m] - rowzx[m] * bias[col] (one load per row and tile)
    int32_t rterm = 0, rzx = 0;
    const bool rowmode = KIND == kOutS32 && a.epi.rowterm != nullptr;
    if (rowmode && m < a.M) {
      rterm = __ldg(a.epi.rowterm + m);
      rzx = __ldg(a.epi.rowzx + m);
    }
    for (int i = 0; i < nmine; ++i) {
      uint32_t va[32];
      int ca = WIDE ? sel * 4 + i : sel + kTcEpiPerQuarter * i;
      int tcol = ca * 32;  // TMEM column of the chunk
      int m_c = m;
      size_t off_c = row_off;
      if (a.rt_G > 1) {
        // row group j = ca / ncols: TMEM columns j * BN.., output rows j * rt_T lower
        const int j = ca / ncols;
        ca -= j * ncols;
        tcol = j * a.BN + ca * 32;
        const int ho = rt_ho0 + j * a.rt_T + ti;
        m_c = (ti < a.rt_T && ho < a.Ho && two < a.Wo) ? 0 : a.M;
        off_c = (static_cast<size_t>(rt_img * a.Ho + ho) * a.Wo + two) * a.ldc;
      }
      tmem_ld_32x32b_x32(tbase + tcol, va);
      tmem_ld_wait();
      if constexpr (KIND == kOutS32) {
        if (rowmode) {
          const int nc = n0 + ca * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int32_t bj = (nc + j < a.N) ? bias[nc + j] : 0;
            va[j] = static_cast<uint32_t>(va[j]) + static_cast<uint32_t>(rterm) -
                    static_cast<uint32_t>(rzx) * static_cast<uint32_t>(bj);
          }
        }
      }
      emit_chunk<KIND, TMA, CL, RES, WIDE>(a, tmC, va, b, m_c, mrow0, off_c, n0 + ca * 32, lane, sbufs, sb, bias,
                                           scale, has_bias && !rowmode, i, i + 1 == nmine);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if constexpr (PAIR)
        mbar_arrive_cluster(mapa_shared(acce0 + 8 * buf, 0));
      else
        mbar_arrive(acce0 + 8 * buf);
    }
    if (++buf == a.nacc) {
      buf = 0;
      acc_ph ^= 1u;
    }
  }
  if (TMA && lane == 0) bulk_wait_group_all();
}

template <int KIND, bool PAIR = false>
__device__ __forceinline__ void epilogue_role(const TcArgs& a, const CUtensorMap* tmC, uint32_t tmem_base,
                                              uint32_t accf0, uint32_t acce0, int warp, int lane,
                                              const int32_t* bias, const float* scale, bool has_bias,
                                              uint8_t* sbufs) {
  // int8 outputs: one compiled variant per clamp form (quant4_s8's CL: the per-element branch
  // stays out of the unrolled loop) and per fused residual add.
#define B200Q_EPI_W(TMA, CL, RES, WIDE)                                                                    \
  epilogue_role_t<KIND, TMA, CL, PAIR, RES, WIDE>(a, tmC, tmem_base, accf0, acce0, warp, lane, bias, scale, \
                                                  has_bias, sbufs)
#define B200Q_EPI(TMA, CL, RES) B200Q_EPI_W(TMA, CL, RES, false)
#define B200Q_EPI_CLW(TMA, RES, WIDE)  \
  if (cl == 4)                         \
    B200Q_EPI_W(TMA, 4, RES, WIDE);    \
  else if (cl == 1)                    \
    B200Q_EPI_W(TMA, 1, RES, WIDE);    \
  else if (cl == 2)                    \
    B200Q_EPI_W(TMA, 2, RES, WIDE);    \
  else                                 \
    B200Q_EPI_W(TMA, 0, RES, WIDE)
#define B200Q_EPI_CL(TMA, RES) B200Q_EPI_CLW(TMA, RES, false)
  if constexpr (KIND != kOutS8) {
    if (a.tma_store)
      B200Q_EPI(true, 0, false);
    else
      B200Q_EPI(false, 0, false);
  } else {
    const int cl = a.default_clamp ? 1 : (a.epi.zp == 0 && a.epi.lo == 0) ? (a.epi.hi >= 127 ? 4 : 2) : 0;
    if (!PAIR && kTcEpiPerQuarter == 2 && a.wide_store) {
      if (a.epi.res) {
        B200Q_EPI_CLW(true, true, !PAIR);
      } else {
        B200Q_EPI_CLW(true, false, !PAIR);
      }
    } else if (a.epi.res) {
      if (a.tma_store) {
        B200Q_EPI_CL(true, true);
      } else {
        B200Q_EPI_CL(false, true);
      }
    } else if (a.tma_store) {
      B200Q_EPI_CL(true, false);
    } else {
      B200Q_EPI_CL(false, false);
    }
  }
#undef B200Q_EPI_CL
#undef B200Q_EPI_CLW
#undef B200Q_EPI
#undef B200Q_EPI_W
}

// Epilogue warps: stage bias / scale in shared memory when they fit, then drain the accumulators.
template <bool PAIR>
__device__ __forceinline__ void run_epilogue(const TcArgs& a, const CUtensorMap* tmC, uint32_t tmem_base,
                                             uint32_t accf0, uint32_t acce0, int warp, int lane, int32_t* s_bias,
                                             float* s_scale, uint8_t* s_out) {
  const bool has_bias = a.epi.bias != nullptr;
  uint8_t* sbufs = s_out + (warp - 2) * 2 *
                              (a.epi.out_kind == kOutS8 ? (a.wide_store ? kEpiStageBytesS8W : kEpiStageBytesS8)
                                                        : kEpiStageBytes);
  if (a.stage_cols > 0) {
    // Copy the per-column bias / scale into shared memory once per CTA (epilogue warps only).
    for (int i = threadIdx.x - 64; i < a.stage_cols; i += kTcEpiWarps * 32) {
      s_bias[i] = (has_bias && i < a.N) ? __ldg(a.epi.bias + i) : 0;
      s_scale[i] = (a.epi.scale && i < a.N) ? __ldg(a.epi.scale + i) : 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kTcEpiWarps * 32) : "memory");
    // s_bias / s_scale derive from the shared-memory window here, so the per-chunk reads
    // compile to shared-memory loads rather than generic ones.
    if (a.epi.out_kind == kOutS8)
      epilogue_role<kOutS8, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, s_bias, s_scale, has_bias, sbufs);
    else if (a.epi.out_kind == kOutS32)
      epilogue_role<kOutS32, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, s_bias, s_scale, has_bias, sbufs);
    else
      epilogue_role<kOutF32, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, s_bias, s_scale, has_bias, sbufs);
  } else {
    if (a.epi.out_kind == kOutS8)
      epilogue_role<kOutS8, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, a.epi.bias, a.epi.scale, has_bias,
                                  sbufs);
    else if (a.epi.out_kind == kOutS32)
      epilogue_role<kOutS32, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, a.epi.bias, a.epi.scale, has_bias,
                                   sbufs);
    else
      epilogue_role<kOutF32, PAIR>(a, tmC, tmem_base, accf0, acce0, warp, lane, a.epi.bias, a.epi.scale, has_bias,
                                   sbufs);
  }
}

// MMA issue of row tiles (mode 2): per tile, 9 taps x KS K-slices of 32 bytes, fully unrolled.
// The operand descriptors are the stage base plus compile-time or per-CTA offsets, so the issuing
// warp spends a few instructions per tcgen05.mma: runtime divisions and 64-bit products in this
// loop cost more than a 64-column MMA itself (~48 SM cycles).  Returns false after a timed-out
// wait (the error flag is already set).
template <int KS>
__device__ __forceinline__ bool rowtile_mma_loop(const TcArgs& a, uint32_t tmem_base, uint64_t rt_desc0,
                                                 uint64_t b_desc0, uint32_t stage_a, uint32_t stage_b,
                                                 uint32_t pl2, uint32_t full0, uint32_t empty0, uint32_t accf0,
                                                 uint32_t acce0) {
  const uint32_t P = static_cast<uint32_t>(a.rt_P);
  const uint32_t bstep = stage_b >> 4;
  const uint32_t idesc = a.idesc;
  int stage = 0, buf = 0;
  uint32_t ph = 0, acc_ph = 0;
  for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x) {
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(acce0 + 8 * buf, acc_ph ^ 1u, a.wait_limit, a.err,
                                                   kDevErrTimeoutMma)))
      return false;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * a.acc_cols);
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(full0 + 8 * stage, ph, a.wait_limit, a.err, kDevErrTimeoutMma)))
      return false;
    const uint64_t ad_s = rt_desc0 + ((stage * stage_a) >> 4);
    for (int gj = 0; gj < a.rt_G; ++gj) {  // row group gj: window rows gj * rt_T lower, TMEM columns gj * BN
      const uint64_t ad_g = ad_s + static_cast<uint64_t>(gj * a.rt_T) * P;
      const uint32_t d_g = d_tmem + static_cast<uint32_t>(gj * a.BN);
#pragma unroll
      for (int tap = 0; tap < 9; ++tap) {
        const uint64_t at = ad_g + static_cast<uint64_t>((tap / 3) * P + (tap % 3));
#pragma unroll
        for (int j = 0; j < KS; ++j)
          tc_mma_i8_elect(d_g, at + static_cast<uint64_t>(j * pl2),
                          b_desc0 + static_cast<uint64_t>(tap * bstep + j * 2), idesc, (tap | j) != 0 ? 1u : 0u);
      }
    }
    tc_commit_elect(empty0 + 8 * stage);
    if (++stage == a.stages) {
      stage = 0;
      ph ^= 1u;
    }
    tc_commit_elect(accf0 + 8 * buf);
    if (++buf == a.nacc) {
      buf = 0;
      acc_ph ^= 1u;
    }
  }
  return true;
}

// MMA issue of the tiled / im2col modes: per K block (one ring stage) KS K-slices of 32 bytes,
// unrolled, with the stage offsets advanced by adds instead of products.  BRES: the weights are
// MMA issue of tap-pair row tiles: R x S taps over 16-channel pixels, S / 2 K = 32 slices per tap
// row (taps s and s + 1), fully unrolled; weights resident (slice kb at kb * stage_b).
template <int R, int S>
__device__ __forceinline__ bool rowtile_pair_loop(const TcArgs& a, uint32_t tmem_base, uint64_t rt_desc0,
                                                  uint64_t b_desc0, uint32_t stage_a, uint32_t stage_b,
                                                  uint32_t full0, uint32_t empty0, uint32_t accf0, uint32_t acce0) {
  const uint32_t P = static_cast<uint32_t>(a.rt_P);
  const uint32_t bstep = stage_b >> 4;
  const uint32_t idesc = a.idesc;
  int stage = 0, buf = 0;
  uint32_t ph = 0, acc_ph = 0;
  for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x) {
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(acce0 + 8 * buf, acc_ph ^ 1u, a.wait_limit, a.err,
                                                   kDevErrTimeoutMma)))
      return false;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * a.acc_cols);
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(full0 + 8 * stage, ph, a.wait_limit, a.err, kDevErrTimeoutMma)))
      return false;
    const uint64_t ad_s = rt_desc0 + ((stage * stage_a) >> 4);
    for (int gj = 0; gj < a.rt_G; ++gj) {  // row group gj: window rows gj * rt_T lower, TMEM columns gj * BN
      const uint64_t ad_g = ad_s + static_cast<uint64_t>(gj * a.rt_T) * P;
      const uint32_t d_g = d_tmem + static_cast<uint32_t>(gj * a.BN);
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int sp = 0; sp < S / 2; ++sp) {
          const int kb = r * (S / 2) + sp;
          tc_mma_i8_elect(d_g, ad_g + static_cast<uint64_t>(r * P + 2 * sp), b_desc0 + static_cast<uint64_t>(kb * bstep),
                          idesc, kb != 0 ? 1u : 0u);
        }
    }
    tc_commit_elect(empty0 + 8 * stage);
    if (++stage == a.stages) {
      stage = 0;
      ph ^= 1u;
    }
    tc_commit_elect(accf0 + 8 * buf);
    if (++buf == a.nacc) {
      buf = 0;
      acc_ph ^= 1u;
    }
  }
  return true;
}

// resident (K block kb of B at kb * stage_b) rather than in the ring.
template <int KS, bool BRES, bool TF32 = false>
__device__ __forceinline__ bool gemm_mma_loop(const TcArgs& a, uint32_t tmem_base, uint64_t a_desc0, uint64_t b_desc0,
                                              uint32_t sa16, uint32_t sb16, uint32_t as16, uint32_t bs16,
                                              uint32_t full0, uint32_t empty0, uint32_t accf0, uint32_t acce0) {
  const uint32_t idesc = a.idesc;
  const int num_kb = a.num_kb, stages = a.stages;
  int stage = 0, buf = 0;
  uint32_t ph = 0, acc_ph = 0, a_off = 0, b_off = 0;
  for (int tile = blockIdx.x; tile < a.total_tiles; tile += gridDim.x) {
    if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(acce0 + 8 * buf, acc_ph ^ 1u, a.wait_limit, a.err,
                                                   kDevErrTimeoutMma)))
      return false;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * a.acc_cols);
    uint32_t bres_off = 0;
    for (int kb = 0; kb < num_kb; ++kb) {
      // The TMA completion on the mbarrier orders the tiles for the tensor core; a tcgen05
      // fence per stage is not needed.
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(full0 + 8 * stage, ph, a.wait_limit, a.err, kDevErrTimeoutMma)))
        return false;
      const uint64_t ad = a_desc0 + a_off;
      const uint64_t bd = b_desc0 + (BRES ? bres_off : b_off);
#pragma unroll
      for (int j = 0; j < KS; ++j) {
        if constexpr (TF32)
          tc_mma_tf32_elect(d_tmem, ad + static_cast<uint64_t>(j * as16), bd + static_cast<uint64_t>(j * bs16), idesc,
                            (kb != 0 || j != 0) ? 1u : 0u);
        else
          tc_mma_i8_elect(d_tmem, ad + static_cast<uint64_t>(j * as16), bd + static_cast<uint64_t>(j * bs16), idesc,
                          (kb != 0 || j != 0) ? 1u : 0u);
      }
      tc_commit_elect(empty0 + 8 * stage);
      bres_off += sb16;
      a_off += sa16;
      b_off += sb16;
      if (++stage == stages) {
        stage = 0;
        ph ^= 1u;
        a_off = 0;
        b_off = 0;
      }
    }
    tc_commit_elect(accf0 + 8 * buf);
    if (++buf == a.nacc) {
      buf = 0;
      acc_ph ^= 1u;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_s8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const TcArgs a,
                      const __grid_constant__ CUtensorMap tmA2) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by pointer arithmetic on the shared window (an integer round trip would
  // turn every later access through these pointers into a generic load / store).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t stage_a = a.mode == 2 ? static_cast<uint32_t>(a.rt_stage) : kTcBM * a.BK;
  const uint32_t stage_b = a.BN * a.BK;
  // Ring of stages: A (+ B unless B is resident).  A resident B holds num_kb blocks after the ring.
  uint8_t* sA = smem;
  uint8_t* sB = smem + a.stages * stage_a;
  const uint32_t b_bytes = a.b_res ? a.num_kb * stage_b : a.stages * stage_b;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + b_bytes);
  // bars: full[stages], empty[stages], acc_full[8], acc_empty[8], drain, b_full, TMEM slot
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + a.stages);
  const uint32_t accf0 = smem_u32(bars + 2 * a.stages);
  const uint32_t acce0 = smem_u32(bars + 2 * a.stages + kTcMaxAcc);
  const uint32_t drain = smem_u32(bars + 2 * a.stages + 2 * kTcMaxAcc);
  const uint32_t b_full = smem_u32(bars + 2 * a.stages + 2 * kTcMaxAcc + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * a.stages + 2 * kTcMaxAcc + 2);
  // bias[stage_cols] then scale[stage_cols], 16-byte aligned, after the barriers
  int32_t* s_bias = reinterpret_cast<int32_t*>(bars + 2 * a.stages + 2 * kTcMaxAcc + 4);
  float* s_scale = reinterpret_cast<float*>(s_bias + a.stage_cols);
  // TMA-store staging: 2 x 4 KiB per epilogue warp, 1024-byte aligned, after the bias / scale copy
  uint8_t* s_out = reinterpret_cast<uint8_t*>(s_scale + a.stage_cols);
  s_out += (1024u - (smem_u32(s_out) & 1023u)) & 1023u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    for (int i = 0; i < a.nacc; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, kTcEpiWarps);
    }
    mbar_init(drain, 1);
    mbar_init(b_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (a.kb_third) tma_prefetch_desc(&tmA2);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Broadcast from lane 0 so the compiler treats the TMEM base as warp-uniform.
  const uint32_t tmem_base = __shfl_sync(0xFFFFFFFFu, *tmem_slot, 0);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t ph = 0;
      uint32_t issued_mask = 0;  // stages that received a load
      uint32_t last_ph = 0;      // parity of the last load into each stage (bit per stage)
      bool ok = true;
      const uint32_t tx = a.mode == 2 ? static_cast<uint32_t>(a.rt_box) : (a.b_res ? stage_a : stage_a + stage_b);
      // One B block (K block kb of N tile n0, batch bb) into shared memory at dB.
      auto load_b = [&](uint32_t dB, uint32_t bar, int kb, int n0, int bb) {
        if (a.conv_b) {
          const int tap = a.mode == 1 ? kb / a.cchunks : 0;
          const int cc = kb - tap * a.cchunks;
          tma_load_3d(dB, &tmB, bar, cc * a.BK, tap, n0);
        } else if (a.b_major == 0) {
          tma_load_3d(dB, &tmB, bar, kb * a.BK, n0, bb);
        } else {
          for (int i = 0; i < a.BN / 128; ++i) tma_load_3d(dB + i * a.BK * 128, &tmB, bar, n0 + 128 * i, kb * a.BK, bb);
        }
      };
      if (a.b_res && blockIdx.x < a.total_tiles) {
        // The whole B of the single N tile, once: the weights of a narrow layer are re-read for
        // every 128-row tile otherwise, and boxes that reach past N or C are slow to fill.
        mbar_arrive_expect_tx(b_full, a.num_kb * stage_b);
        for (int kb = 0; kb < a.num_kb; ++kb) load_b(smem_u32(sB + kb * stage_b), b_full, kb, 0, 0);
      }
      // Row tiles: one window load per tile (all taps, all channels); tiles enumerate
      // (image, block of rt_T output rows).
      const int rt_tb = a.rt_T * a.rt_G;  // output rows per tile
      TileWalk rw(a.mode == 2 ? static_cast<int>(blockIdx.x) : 0, gridDim.x, 1 << 30,
                  a.mode == 2 ? (a.Ho + rt_tb - 1) / rt_tb : 1, 1);
      for (int tile = blockIdx.x; tile < a.total_tiles && ok && a.mode == 2; tile += gridDim.x, rw.next()) {
        const int img = rw.b;
        const int ho0 = rw.mt * rt_tb;
        if (!mbar_wait_bounded(empty0 + 8 * stage, ph ^ 1u, a.wait_limit, a.err, kDevErrTimeoutProducer)) {
          ok = false;
          break;
        }
        const uint32_t fb = full0 + 8 * stage;
        mbar_arrive_expect_tx(fb, tx);
        if (a.rt_wide)
          tma_load_3d(smem_u32(sA + stage * stage_a), &tmA, fb, 2 * a.rt_x0, ho0 + a.rt_y0, img);
        else
          tma_load_5d(smem_u32(sA + stage * stage_a), &tmA, fb, 0, a.rt_x0, ho0 + a.rt_y0, 0, img);
        issued_mask |= 1u << stage;
        last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
        if (++stage == a.stages) {
          stage = 0;
          ph ^= 1u;
        }
      }
      TileWalk tw(blockIdx.x, gridDim.x, a.batch, a.m_tiles, a.n_tiles);
      for (int tile = blockIdx.x; tile < a.total_tiles && ok && a.mode != 2; tile += gridDim.x, tw.next()) {
        const int b = tw.b, mt = tw.mt, nt = tw.nt;
        const int m0 = mt * kTcBM, n0 = nt * a.BN;
        int img = 0, wbase = 0, hbase = 0;
        if (a.mode == 1) {
          const int hw = a.Ho * a.Wo;
          img = m0 / hw;
          const int r0 = m0 - img * hw;
          const int ho = r0 / a.Wo;
          const int wo = r0 - ho * a.Wo;
          wbase = wo * a.stride_w - a.pad_w;
          hbase = ho * a.stride_h - a.pad_h;
        }
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!mbar_wait_bounded(empty0 + 8 * stage, ph ^ 1u, a.wait_limit, a.err, kDevErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          mbar_arrive_expect_tx(fb, tx);
          const uint32_t dA = smem_u32(sA + stage * stage_a);
          const uint32_t dB = smem_u32(sB + stage * stage_b);
          if (a.mode == 1) {
            // fp32 (tf32 split) convs walk the taps three times: thirds 0 and 1 read the hi copy
            // of the input (tmA), third 2 the lo copy (tmA2)
            const int third = a.kb_third ? kb / a.kb_third : 0;
            const int kk = kb - third * a.kb_third;
            const int tap = kk / a.cchunks;
            const int cc = kk - tap * a.cchunks;
            const int r = tap / a.S;
            const int s = tap - r * a.S;
            // grouped fp32 convs: batch item b is group b, whose channels start grp_bytes later
            tma_load_im2col_4d(dA, third == 2 ? &tmA2 : &tmA, fb, cc * a.BK + b * a.grp_bytes, wbase, hbase, img,
                               static_cast<uint16_t>(s * a.dil_w), static_cast<uint16_t>(r * a.dil_h));
          } else if (a.a_major == 0) {
            tma_load_3d(dA, &tmA, fb, kb * a.BK, m0, b);
          } else {
            tma_load_3d(dA, &tmA, fb, m0, kb * a.BK, b);
          }
          if (a.b_packed)
            bulk_load(dB, a.b_packed + (static_cast<size_t>(nt) * a.num_kb + kb) * stage_b, stage_b, fb);
          else if (!a.b_res)
            load_b(dB, fb, kb, n0, a.b_batched ? b : 0);
          issued_mask |= 1u << stage;
          last_ph = (last_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == a.stages) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA exits.
        for (int i = 0; i < a.stages; ++i)
          if (issued_mask & (1u << i))
            mbar_wait_bounded(full0 + 8 * i, (last_ph >> i) & 1u, a.wait_limit, a.err, kDevErrTimeoutProducer);
        if (a.b_res) mbar_wait_bounded(b_full, 0, a.wait_limit, a.err, kDevErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    {
      // ----------------------------------------------------------------- MMA
      // The whole warp runs the loop converged; an elected lane issues each tcgen05 instruction.
      bool ok = true;
      const uint32_t a_layout = a.a_major == 0 ? kmajor_layout(a.BK) : 2u;
      const uint32_t b_layout = a.b_major == 0 ? kmajor_layout(a.BK) : 2u;
      const uint32_t a_lbo = a.a_major == 0 ? 16u : static_cast<uint32_t>(a.BK) * 128u;
      const uint32_t a_sbo = a.a_major == 0 ? 8u * a.BK : 1024u;
      const uint32_t b_lbo = a.b_major == 0 ? 16u : static_cast<uint32_t>(a.BK) * 128u;
      const uint32_t b_sbo = a.b_major == 0 ? 8u * a.BK : 1024u;
      const uint32_t a_step = a.a_major == 0 ? 32u : 4096u;  // bytes per K=32 slice
      const uint32_t b_step = a.b_major == 0 ? 32u : 4096u;
      const int ksteps = a.BK / 32;
      // Stage-0 descriptors; stage / K-slice offsets are added to the 14-bit start-address field
      // (shared addresses stay below 256 KiB, so the add never carries out of the field).
      const uint64_t a_desc0 = make_smem_desc(smem_u32(sA), a_lbo, a_sbo, a_layout);
      const uint64_t b_desc0 = make_smem_desc(smem_u32(sB), b_lbo, b_sbo, b_layout);
      if (a.b_res && blockIdx.x < a.total_tiles)
        ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(b_full, 0, a.wait_limit, a.err, kDevErrTimeoutMma));
      // Row tiles: A in the no-swizzle K-major layout [C/16][pixel][16 B] (SBO = 8 pixels, LBO =
      // one channel-chunk plane); tap (r, s) is the same window started (r * P + s) pixels later.
      const uint64_t rt_desc0 = make_smem_desc(smem_u32(sA), static_cast<uint32_t>(a.rt_plane), 128u, 0u);
      if (ok && a.mode == 2 && a.rt_pairs) {
#define B200Q_PAIR_MMA(R, S) \
  ok = rowtile_pair_loop<R, S>(a, tmem_base, rt_desc0, b_desc0, stage_a, stage_b, full0, empty0, accf0, acce0)
        const int rs = a.rt_R * 8 + a.rt_S;
        if (rs == 4 * 8 + 4) B200Q_PAIR_MMA(4, 4);
        else if (rs == 4 * 8 + 2) B200Q_PAIR_MMA(4, 2);
        else if (rs == 3 * 8 + 4) B200Q_PAIR_MMA(3, 4);
        else if (rs == 3 * 8 + 2) B200Q_PAIR_MMA(3, 2);
        else if (rs == 2 * 8 + 4) B200Q_PAIR_MMA(2, 4);
        else B200Q_PAIR_MMA(2, 2);
#undef B200Q_PAIR_MMA
      } else if (ok && a.mode == 2) {
        const uint32_t pl2 = static_cast<uint32_t>(a.rt_plane) >> 3;  // two channel-chunk planes
        switch (a.BK) {
          case 32:
            ok = rowtile_mma_loop<1>(a, tmem_base, rt_desc0, b_desc0, stage_a, stage_b, pl2, full0, empty0, accf0, acce0);
            break;
          case 64:
            ok = rowtile_mma_loop<2>(a, tmem_base, rt_desc0, b_desc0, stage_a, stage_b, pl2, full0, empty0, accf0, acce0);
            break;
          default:
            ok = rowtile_mma_loop<4>(a, tmem_base, rt_desc0, b_desc0, stage_a, stage_b, pl2, full0, empty0, accf0, acce0);
            break;
        }
      }
      if (ok && a.mode != 2) {
        const uint32_t sa16 = stage_a >> 4, sb16 = stage_b >> 4, as16 = a_step >> 4, bs16 = b_step >> 4;
#define B200Q_GEMM_MMA(KS, BRES)                                                                              \
  ok = gemm_mma_loop<KS, BRES>(a, tmem_base, a_desc0, b_desc0, sa16, sb16, as16, bs16, full0, empty0, accf0, acce0)
        if (a.tf32) {
          // fp32 GEMMs (3 x TF32 split operands): tiled mode, 128-byte K blocks, B in the ring
          ok = gemm_mma_loop<4, false, true>(a, tmem_base, a_desc0, b_desc0, sa16, sb16, as16, bs16, full0, empty0,
                                             accf0, acce0);
        } else if (a.b_res) {
          if (ksteps == 4) B200Q_GEMM_MMA(4, true);
          else if (ksteps == 2) B200Q_GEMM_MMA(2, true);
          else B200Q_GEMM_MMA(1, true);
        } else {
          if (ksteps == 4) B200Q_GEMM_MMA(4, false);
          else if (ksteps == 2) B200Q_GEMM_MMA(2, false);
          else B200Q_GEMM_MMA(1, false);
        }
#undef B200Q_GEMM_MMA
      }
      // Wait for every MMA issued by this warp before TMEM is released.
      tc_commit_elect(drain);
      mbar_wait_bounded(drain, 0, a.wait_limit, a.err, kDevErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    run_epilogue<false>(a, &tmC, tmem_base, accf0, acce0, warp, lane, s_bias, s_scale, s_out);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// 2-SM variant for large tiled GEMMs (mode 0, K-major A and B, BN = 256): a cluster of two CTAs
// computes a 256 x 256 tile with M = 256 tcgen05 MMAs issued by the leader (rank 0).  Each CTA
// loads its own 128 rows of A and 128 rows of B (half the B bytes per SM of the one-CTA tile);
// both loads count on the leader's full barrier; the leader's commits arrive on the empty and
// accumulator-full barriers of both CTAs; the peer's epilogue warps release accumulators on the
// leader's barrier.  No TMA multicast.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    tc_gemm_s8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmC, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t stage_a = kTcBM * a.BK;
  const uint32_t stage_b = (a.BN / 2) * a.BK;
  uint8_t* sA = smem;
  uint8_t* sB = smem + a.stages * stage_a;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + a.stages * stage_b);
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + a.stages);
  const uint32_t accf0 = smem_u32(bars + 2 * a.stages);
  const uint32_t acce0 = smem_u32(bars + 2 * a.stages + kTcMaxAcc);
  const uint32_t drain = smem_u32(bars + 2 * a.stages + 2 * kTcMaxAcc);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * a.stages + 2 * kTcMaxAcc + 2);
  int32_t* s_bias = reinterpret_cast<int32_t*>(bars + 2 * a.stages + 2 * kTcMaxAcc + 4);
  float* s_scale = reinterpret_cast<float*>(s_bias + a.stage_cols);
  uint8_t* s_out = reinterpret_cast<uint8_t*>(s_scale + a.stage_cols);
  s_out += (1024u - (smem_u32(s_out) & 1023u)) & 1023u;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int unit = static_cast<int>(blockIdx.x >> 1);
  const int nunits = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.stages; ++i) {
      mbar_init(full0 + 8 * i, 2);  // one arrive.expect_tx per CTA of the pair
      mbar_init(empty0 + 8 * i, 1);
    }
    for (int i = 0; i < a.nacc; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 2 * kTcEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = __shfl_sync(0xFFFFFFFFu, *tmem_slot, 0);
  const int tiles_per_batch = a.m_tiles * a.n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer (both CTAs)
      int stage = 0;
      uint32_t ph = 0;
      const uint32_t tx = stage_a + stage_b;
      const uint32_t full_leader = mapa_shared(full0, 0);
      for (int tile = unit; tile < a.total_tiles; tile += nunits) {
        const int b = tile / tiles_per_batch;
        const int rem = tile - b * tiles_per_batch;
        const int mt = rem / a.n_tiles;
        const int nt = rem - mt * a.n_tiles;
        const int m0 = mt * 2 * kTcBM + rank * kTcBM;
        const int nb0 = nt * a.BN + rank * (a.BN / 2);
        const int bb = a.b_batched ? b : 0;
        bool ok = true;
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!mbar_wait_bounded(empty0 + 8 * stage, ph ^ 1u, a.wait_limit, a.err, kDevErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_leader + 8 * stage;
          // Relaxed: the bytes are ordered by the TMA's own complete_tx; a release at cluster scope
          // here cost half the throughput.
          if (rank == 0)
            mbar_arrive_expect_tx(full0 + 8 * stage, tx);
          else
            mbar_arrive_expect_tx_cluster_relaxed(fb, tx);
          tma_load_3d_pair(smem_u32(sA + stage * stage_a), &tmA, fb, kb * a.BK, m0, b);
          if (a.b_major == 0)
            tma_load_3d_pair(smem_u32(sB + stage * stage_b), &tmB, fb, kb * a.BK, nb0, bb);
          else  // MN-major B (bmm NN): one 128-column box of BK K rows
            tma_load_3d_pair(smem_u32(sB + stage * stage_b), &tmB, fb, nb0, kb * a.BK, bb);
          if (++stage == a.stages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ----------------------------------------------------------------- MMA (leader only)
      int stage = 0;
      uint32_t ph = 0;
      int buf = 0;
      uint32_t acc_ph = 0;
      bool ok = true;
      const uint32_t layout = kmajor_layout(a.BK);
      const uint64_t a_desc0 = make_smem_desc(smem_u32(sA), 16u, 8u * a.BK, layout);
      // MN-major B: this CTA's 128 columns are one 128-byte swizzle atom wide, K rows 128 bytes
      // apart (8-row groups 1024 bytes apart); a K = 32 slice is 32 rows = 4096 bytes on.
      const bool bmn = a.b_major != 0;
      const uint64_t b_desc0 = bmn ? make_smem_desc(smem_u32(sB), static_cast<uint32_t>(a.BK) * 128u, 1024u, 2u)
                                   : make_smem_desc(smem_u32(sB), 16u, 8u * a.BK, layout);
      const int ksteps = a.BK / 32;
      for (int tile = unit; tile < a.total_tiles && ok; tile += nunits) {
        if (!__all_sync(0xFFFFFFFFu,
                        mbar_wait_bounded(acce0 + 8 * buf, acc_ph ^ 1u, a.wait_limit, a.err, kDevErrTimeoutMma))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * a.acc_cols);
        for (int kb = 0; kb < a.num_kb; ++kb) {
          if (!__all_sync(0xFFFFFFFFu,
                          mbar_wait_bounded(full0 + 8 * stage, ph, a.wait_limit, a.err, kDevErrTimeoutMma))) {
            ok = false;
            break;
          }
          const uint64_t ad_s = a_desc0 + ((stage * stage_a) >> 4);
          const uint64_t bd_s = b_desc0 + ((stage * stage_b) >> 4);
          if (bmn) {
            for (int j = 0; j < ksteps; ++j)
              tc_mma_i8_pair_elect(d_tmem, ad_s + 2 * j, bd_s + 256 * j, a.idesc, (kb | j) != 0 ? 1u : 0u);
          } else if (ksteps == 4) {
            tc_mma_i8_pair_kblock4(d_tmem, ad_s, bd_s, a.idesc, kb != 0 ? 1u : 0u);
          } else {
            for (int j = 0; j < ksteps; ++j)
              tc_mma_i8_pair_elect(d_tmem, ad_s + 2 * j, bd_s + 2 * j, a.idesc, (kb | j) != 0 ? 1u : 0u);
          }
          tc_commit_pair_elect(empty0 + 8 * stage);
          if (++stage == a.stages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_elect(accf0 + 8 * buf);
        if (++buf == a.nacc) {
          buf = 0;
          acc_ph ^= 1u;
        }
      }
      tc_commit_pair_elect(drain);
      mbar_wait_bounded(drain, 0, a.wait_limit, a.err, kDevErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------- epilogue (both CTAs)
    run_epilogue<true>(a, &tmC, tmem_base, accf0, acce0, warp, lane, s_bias, s_scale, s_out);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no remote arrive or MMA into this CTA's TMEM after this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, a.tmem_cols);
  }
}

// Failure-path probe: one thread waits on a barrier nobody completes, with a small limit.
__global__ void wait_timeout_probe_kernel(long long limit, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
    mbar_wait_bounded(smem_u32(&bar), 0, limit, err, kDevErrTimeoutProbe);
  }
}

// Prepack conv weights w[N][taps][C] (int8, C % 16 == 0, 16-byte aligned) into the shared-memory
// images of the B operand (BN rows x 128-byte K blocks, SWIZZLE_128B: 16-byte unit u of row r at
// unit u ^ (r % 8)), one image per (N tile, K block), K block kb = tap * cchunks + cc covering
// channels [cc * 128, cc * 128 + 128) of tap `tap`; rows past N and channels past C are zero, as
// the tensor map's out-of-bounds fill gives.  One thread writes one 16-byte unit.
__global__ void pack_b_stages_kernel(const int8_t* __restrict__ w, int8_t* __restrict__ out, int N, int taps, int C,
                                     int cchunks, int num_kb, int BN, long long units) {
  for (long long u = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; u < units;
       u += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int pos = static_cast<int>(u & 7);
    const long long rowi = u >> 3;  // (nt * num_kb + kb) * BN + row
    const int row = static_cast<int>(rowi % BN);
    const long long blk = rowi / BN;
    const int kb = static_cast<int>(blk % num_kb);
    const int nt = static_cast<int>(blk / num_kb);
    const int unit = pos ^ (row & 7);
    const int tap = kb / cchunks;
    const int ch = (kb - tap * cchunks) * 128 + unit * 16;
    const int n = nt * BN + row;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (n < N && ch < C)
      v = __ldg(reinterpret_cast<const uint4*>(w + (static_cast<size_t>(n) * taps + tap) * C + ch));
    reinterpret_cast<uint4*>(out)[u] = v;
  }
}

// Pixel-grouped 1x1 conv: G consecutive pixels are one GEMM row of G * C channels, and the
// weights become the block-diagonal [G * K][G * C] matrix (block g maps pixel g's channels to its
// K outputs), so the output rows [G * K] are the same bytes as G NHWC output pixels.  Also expands
// bias / scale to G * K columns (entry j = entry j % K; null stays null).
__global__ void group_weights_kernel(const int8_t* __restrict__ w, int8_t* __restrict__ wg, int32_t* __restrict__ bg,
                                     float* __restrict__ sg, const int32_t* __restrict__ bias,
                                     const float* __restrict__ scale, int K, int C, int G) {
  const long long total = static_cast<long long>(G) * K * G * C;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / (static_cast<long long>(G) * C);
    const int col = static_cast<int>(i - row * G * C);
    const int gr = static_cast<int>(row / K), k = static_cast<int>(row - static_cast<long long>(gr) * K);
    const int gc = col / C, c = col - gc * C;
    wg[i] = gr == gc ? w[static_cast<size_t>(k) * C + c] : static_cast<int8_t>(0);
    if (col == 0) {
      if (bias) bg[row] = bias[k];
      if (scale) sg[row] = scale[k];
    }
  }
}

}  // namespace b200q
