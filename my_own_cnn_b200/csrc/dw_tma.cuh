// Depthwise 3x3 int8 conv (groups == C == K) with TMA-staged input tiles, for int8 outputs.
//
// The layer is HBM-bound (9 MACs per output byte), so the kernel is built around keeping enough
// bytes in flight: a persistent CTA walks tiles (channel slab, image, block of output rows, block of
// output columns) and, for each, one elected thread loads the tile's whole input window (CB
// channels x wbox columns x rows_in rows) with a single 4-D TMA box into a ring of shared-memory
// stages, issued `stages - 1` tiles ahead.  Padding is the TMA's zero fill (a box may start at a
// negative row / column), so no thread branches on borders.
//
// Roles: warp 8 is the producer (one lane issues the boxes, waiting on each slot's `empty` barrier);
// warps 0-7 compute and release a slot with one arrive per warp, so no block-wide barrier sits
// between tiles.
//
// Compute: thread = 8 channels of one output column, walking down its rows.  Per input row it
// reads the three taps' 8-byte words from shared memory (consecutive lanes read consecutive 8-byte
// chunks: conflict-free for stride 1), byte-transposes them so one word holds one channel's three
// taps of that row (transpose4x4_bytes: 6 prmt per 4 channels), and keeps the last three rows'
// words in registers.  An output is then three dp4a per channel against the channel's filter rows
// (w[r][0..2] in bytes 0..2, byte 3 zero; the bias is the first dp4a's accumulator, the same
// int32 wrap-around add), followed by the fused requantization in one of three compiled clamp
// forms.  A stride-1 walk transposes one new input row per output row, a stride-2 walk two; the
// three window rows rotate through register sets instead of being copied.
#pragma once
#include "common.cuh"
#include "ptx.cuh"
#include "simt.cuh"

namespace b200q {

struct DwPlan {
  int CB;          // channels per slab (multiple of 16, divides C, <= 256: the TMA box limit)
  int g8;          // CB / 8 threads across a slab
  int TW;          // output columns per tile
  int RG;          // row groups: threads of one column split the tile's rows into RG runs
  int rpt;         // output rows per thread (TH = RG * rpt)
  int TH;          // output rows per tile
  int rows_in;     // input rows per box: (TH - 1) * stride + 3
  int wbox;        // input columns per box: (TW - 1) * stride + 3
  int box_bytes;   // CB * wbox * rows_in
  int stage;       // ring stage bytes (box rounded up to 1024)
  int stages;      // ring depth
  int slabs, row_tiles, col_tiles;
  int total;       // tiles
  long long wait_limit;
  int* err;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Tile t -> (slab, image, row block, column block); slab outermost so a persistent CTA keeps the
// same filter slab (and its weights in registers) over consecutive tiles.
struct DwTile {
  int slab, n, rt, ct;
};
__device__ __forceinline__ DwTile dw_tile(const DwPlan& p, int n_img, int t) {
  DwTile d;
  d.ct = t % p.col_tiles;
  t /= p.col_tiles;
  d.rt = t % p.row_tiles;
  t /= p.row_tiles;
  d.n = t % n_img;
  d.slab = t / n_img;
  return d;
}

// Channel words of one input row: bytes of pixel columns s = 0, 1, 2 regrouped per channel
// (channel j of the 8: word j holds taps s = 0, 1, 2 in bytes 0..2, byte 3 zero).
__device__ __forceinline__ void dw_row_words(const uint2 a, const uint2 b, const uint2 c, uint32_t (&t)[8]) {
  transpose4x4_bytes(a.x, b.x, c.x, 0u, t[0], t[1], t[2], t[3]);
  transpose4x4_bytes(a.y, b.y, c.y, 0u, t[4], t[5], t[6], t[7]);
}

// int8 codes of 8 channels from their int32 sums t (bias included): p = fl(t) * scale, then
// CL 1: the saturating pack alone clamps (bounds [-128, 127], zero point 0);
// CL 2: clamp in floats to [0, hi] before the conversion (zero point 0, lower bound 0: ReLU /
//       ReLU6; max(NaN, 0) = 0 keeps rint_sat's NaN rule, and integer bounds commute with rounding);
// CL 0: clamp(rint_sat(p), lo - zp, hi - zp) + zp in integers (any bounds and zero point).
template <int CL>
__device__ __forceinline__ uint2 dw_quant8(const int32_t (&t)[8], const float (&sc)[8], const Epilogue& e,
                                           float hi_f) {
  int r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float f = __fmul_rn(__int2float_rn(t[j]), sc[j]);
    if constexpr (CL == 2) f = fminf(fmaxf(f, 0.0f), hi_f);
    r[j] = __float2int_rn(f);
    if constexpr (CL == 0) r[j] = min(max(r[j], e.lo - e.zp), e.hi - e.zp) + e.zp;
  }
  if constexpr (CL == 0) {
    return make_uint2(__byte_perm(__byte_perm(r[0], r[1], 0x0040), __byte_perm(r[2], r[3], 0x0040), 0x5410),
                      __byte_perm(__byte_perm(r[4], r[5], 0x0040), __byte_perm(r[6], r[7], 0x0040), 0x5410));
  } else {
    uint32_t lo, hi, a, b;
    asm("cvt.pack.sat.s8.s32.b32 %0, %2, %1, 0;" : "=r"(a) : "r"(r[2]), "r"(r[3]));
    asm("cvt.pack.sat.s8.s32.b32 %0, %2, %1, %3;" : "=r"(lo) : "r"(r[0]), "r"(r[1]), "r"(a));
    asm("cvt.pack.sat.s8.s32.b32 %0, %2, %1, 0;" : "=r"(b) : "r"(r[6]), "r"(r[7]));
    asm("cvt.pack.sat.s8.s32.b32 %0, %2, %1, %3;" : "=r"(hi) : "r"(r[4]), "r"(r[5]), "r"(b));
    return make_uint2(lo, hi);
  }
}

// Warp 8 is the TMA producer (one elected lane), warps 0-7 compute.  Ring slot s has a `full`
// barrier (TMA bytes) and an `empty` barrier (one arrive per compute warp when it has read the
// slot), so warps move on to the next tile without a block-wide barrier.
constexpr int kDwComputeThreads = 256;
constexpr int kDwThreads = kDwComputeThreads + 32;

template <int S, int CL>
__global__ void __launch_bounds__(kDwThreads, 2) dw_tma_s8_kernel(const __grid_constant__ CUtensorMap tmx,
                                                                 int8_t* __restrict__ y, const int8_t* __restrict__ w,
                                                                 ConvGeom g, Epilogue e, DwPlan p) {
  extern __shared__ __align__(1024) uint8_t dw_smem[];
  __shared__ __align__(8) uint64_t bars[16];  // full[0..7], empty[8..15]
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dw_smem) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 64;
  // A contiguous run of tiles per CTA (slab outermost): the CTA reloads its filter slab only at
  // the run's slab boundaries instead of every few tiles of a grid-strided walk.
  const int per_cta = (p.total + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int t_begin = min(p.total, static_cast<int>(blockIdx.x) * per_cta);
  const int t_end = min(p.total, t_begin + per_cta);
  if (tid == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, kDwComputeThreads / 32);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == kDwComputeThreads / 32) {
    // ---- producer: one lane issues each tile's window box once its slot is free
    if ((tid & 31) == 0) {
      tma_prefetch_desc(&tmx);
      int it = 0;
      for (int t = t_begin; t < t_end; ++t, ++it) {
        const int slot = it % p.stages;
        if (it >= p.stages &&
            !mbar_wait_bounded(empty0 + 8 * slot, static_cast<uint32_t>(((it / p.stages) - 1) & 1), p.wait_limit,
                               p.err, kDevErrTimeoutDw))
          return;
        const DwTile d = dw_tile(p, g.n, t);
        const uint32_t bar = full0 + 8 * slot;
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(p.box_bytes));
        tma_load_4d(ring_u32 + slot * p.stage, &tmx, bar, d.slab * p.CB, d.ct * p.TW * S - g.pad_w,
                    d.rt * p.TH * S - g.pad_h, d.n);
      }
    }
    return;
  }
  // ---- compute warps
  const int g8i = tid % p.g8;
  const int col = (tid / p.g8) % p.TW;
  const int rg = tid / (p.g8 * p.TW);
  const bool active = rg < p.RG;
  const float hi_f = static_cast<float>(e.hi);
  int cur_slab = -1;
  uint32_t wr[8][3];
  int32_t bias[8];
  float scl[8];
  int it = 0;
  for (int t = t_begin; t < t_end; ++t, ++it) {
    const int slot = it % p.stages;
    const DwTile d = dw_tile(p, g.n, t);
    if (active && d.slab != cur_slab) {
      cur_slab = d.slab;
      const int c0 = d.slab * p.CB + g8i * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int8_t* wp = w + static_cast<size_t>(c0 + j) * 9;
#pragma unroll
        for (int r = 0; r < 3; ++r)
          wr[j][r] = static_cast<uint32_t>(static_cast<uint8_t>(__ldg(wp + 3 * r))) |
                     (static_cast<uint32_t>(static_cast<uint8_t>(__ldg(wp + 3 * r + 1))) << 8) |
                     (static_cast<uint32_t>(static_cast<uint8_t>(__ldg(wp + 3 * r + 2))) << 16);
        bias[j] = e.bias ? __ldg(e.bias + c0 + j) : 0;
        scl[j] = __ldg(e.scale + c0 + j);
      }
    }
    if (!mbar_wait_bounded(full0 + 8 * slot, static_cast<uint32_t>((it / p.stages) & 1), p.wait_limit, p.err,
                           kDevErrTimeoutDw))
      return;
    const int wo = d.ct * p.TW + col;
    const int r0 = rg * p.rpt;  // first output row of this thread, tile-relative
    const int ho0 = d.rt * p.TH + r0;
    const int rows = (active && wo < g.wo) ? min(p.rpt, g.ho - ho0) : 0;
    if (rows > 0) {
      const int pitch = p.wbox * p.CB;  // bytes per staged input row
      const uint8_t* rp = ring + slot * p.stage + (col * S) * p.CB + g8i * 8 + (r0 * S) * pitch;
      int8_t* yp = y + ((static_cast<size_t>(d.n) * g.ho + ho0) * g.wo + wo) * g.c + d.slab * p.CB + g8i * 8;
      const size_t ystep = static_cast<size_t>(g.wo) * g.c;
      auto row_words = [&](uint32_t (&tw)[8]) {
        dw_row_words(*reinterpret_cast<const uint2*>(rp), *reinterpret_cast<const uint2*>(rp + p.CB),
                     *reinterpret_cast<const uint2*>(rp + 2 * p.CB), tw);
        rp += pitch;
      };
      // one output row from the window rows (a, b, c): bias as the first dp4a's accumulator
      auto emit = [&](const uint32_t (&a)[8], const uint32_t (&b)[8], const uint32_t (&c)[8]) {
        int32_t acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int v = __dp4a(static_cast<int>(a[j]), static_cast<int>(wr[j][0]), bias[j]);
          v = __dp4a(static_cast<int>(b[j]), static_cast<int>(wr[j][1]), v);
          acc[j] = __dp4a(static_cast<int>(c[j]), static_cast<int>(wr[j][2]), v);
        }
        *reinterpret_cast<uint2*>(yp) = dw_quant8<CL>(acc, scl, e, hi_f);
        yp += ystep;
      };
      // The window rotates through three register sets (period 3), so no row is copied:
      // stride 1: output i reads rows (i, i+1, i+2) and loads only row i+2;
      // stride 2: output i reads rows (2i, 2i+1, 2i+2) and loads rows 2i+1 and 2i+2.
      uint32_t x0[8], x1[8], x2[8];
      row_words(x0);
      if constexpr (S == 1) {
        row_words(x1);
        for (int i = 0;;) {
          row_words(x2); emit(x0, x1, x2); if (++i == rows) break;
          row_words(x0); emit(x1, x2, x0); if (++i == rows) break;
          row_words(x1); emit(x2, x0, x1); if (++i == rows) break;
        }
      } else {
        for (int i = 0;;) {
          row_words(x1); row_words(x2); emit(x0, x1, x2); if (++i == rows) break;
          row_words(x0); row_words(x1); emit(x2, x0, x1); if (++i == rows) break;
          row_words(x2); row_words(x0); emit(x1, x2, x0); if (++i == rows) break;
        }
      }
    }
    // this warp has read the slot: one arrive per warp frees it for the producer
    __syncwarp();
    if ((tid & 31) == 0) mbar_arrive(empty0 + 8 * slot);
  }
}

}  // namespace b200q
