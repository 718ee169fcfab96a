// Depthwise 3x3 int8 conv (groups == C == K) with TMA-staged input tiles, for int8 outputs.
//
// The layer is HBM-bound (9 MACs per output byte), so the kernel is built around keeping enough
// bytes in flight: a persistent CTA walks tiles (channel slab, image, block of output rows, block of
// output columns) and, for each, one elected thread loads the tile's whole input window (CB
// channels x wbox columns x rows_in rows) with a single 4-D TMA box into a ring of shared-memory
// stages, issued `stages - 1` tiles ahead.  Padding is the TMA's zero fill (a box may start at a
// negative row / column), so no thread branches on borders.
//
// Compute: thread = 8 channels of one output column, walking down its rows.  Per input row it
// reads the three taps' 8-byte words from shared memory (consecutive lanes read consecutive 8-byte
// chunks: conflict-free for stride 1), byte-transposes them so one word holds one channel's three
// taps of that row (transpose4x4_bytes: 6 prmt per 4 channels), and keeps the last three rows'
// words in registers.  An output is then three dp4a per channel against the channel's filter rows
// (w[r][0..2] in bytes 0..2, byte 3 zero), followed by the fused requantization.  A stride-1 walk
// transposes one new input row per output row, a stride-2 walk two.
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

template <int S>
__global__ void __launch_bounds__(256) dw_tma_s8_kernel(const __grid_constant__ CUtensorMap tmx, int8_t* __restrict__ y,
                                                       const int8_t* __restrict__ w, ConvGeom g, Epilogue e, DwPlan p) {
  extern __shared__ __align__(1024) uint8_t dw_smem[];
  __shared__ __align__(8) uint64_t bars[8];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dw_smem) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t bar0 = smem_u32(bars);
  if (tid == 0) {
    for (int i = 0; i < p.stages; ++i) mbar_init(bar0 + 8 * i, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // this thread's place in a tile
  const int g8i = tid % p.g8;
  const int col = (tid / p.g8) % p.TW;
  const int rg = tid / (p.g8 * p.TW);
  const bool active = rg < p.RG;
  const int stride = S;

  auto issue = [&](int t, int slot) {
    const DwTile d = dw_tile(p, g.n, t);
    const uint32_t bar = bar0 + 8 * slot;
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(p.box_bytes));
    tma_load_4d(ring_u32 + slot * p.stage, &tmx, bar, d.slab * p.CB, d.ct * p.TW * stride - g.pad_w,
                d.rt * p.TH * stride - g.pad_h, d.n);
  };
  // prologue: the first stages - 1 tiles of this CTA
  if (tid == 0) {
    tma_prefetch_desc(&tmx);
    for (int i = 0; i < p.stages - 1; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      if (t < p.total) issue(t, i);
    }
  }
  int cur_slab = -1;
  uint32_t wr[8][3];
  int32_t bias[8];
  float scl[8];
  int it = 0;
  for (int t = blockIdx.x; t < p.total; t += gridDim.x, ++it) {
    const int slot = it % p.stages;
    // keep stages - 1 loads in flight: the slot refilled here was last read in iteration it - 1,
    // which every thread finished before the __syncthreads that closed it
    if (tid == 0) {
      const int tn = t + (p.stages - 1) * gridDim.x;
      if (tn < p.total) {
        fence_proxy_async_smem();
        issue(tn, (it + p.stages - 1) % p.stages);
      }
    }
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
    if (!mbar_wait_bounded(bar0 + 8 * slot, static_cast<uint32_t>((it / p.stages) & 1), p.wait_limit, p.err,
                           kDevErrTimeoutDw))
      return;
    const int wo = d.ct * p.TW + col;
    if (active && wo < g.wo) {
      const uint8_t* st = ring + slot * p.stage;
      const int pitch = p.wbox * p.CB;  // bytes per staged input row
      const uint8_t* cp = st + (col * stride) * p.CB + g8i * 8;
      const int r0 = rg * p.rpt;  // first output row of this thread, tile-relative
      const int ho0 = d.rt * p.TH + r0;
      int rows = min(p.rpt, g.ho - ho0);
      uint32_t t0[8], t1[8], t2[8];
      // input rows r0 * stride + {0, 1} prime the window
      {
        const uint8_t* rp = cp + (r0 * stride) * pitch;
        dw_row_words(*reinterpret_cast<const uint2*>(rp), *reinterpret_cast<const uint2*>(rp + p.CB),
                     *reinterpret_cast<const uint2*>(rp + 2 * p.CB), t0);
        rp += pitch;
        dw_row_words(*reinterpret_cast<const uint2*>(rp), *reinterpret_cast<const uint2*>(rp + p.CB),
                     *reinterpret_cast<const uint2*>(rp + 2 * p.CB), t1);
      }
      int8_t* yp = y + ((static_cast<size_t>(d.n) * g.ho + ho0) * g.wo + wo) * g.c + d.slab * p.CB + g8i * 8;
      const size_t ystep = static_cast<size_t>(g.wo) * g.c;
      const uint8_t* rp = cp + (r0 * stride + 2) * pitch;
      for (int i = 0; i < rows; ++i) {
        dw_row_words(*reinterpret_cast<const uint2*>(rp), *reinterpret_cast<const uint2*>(rp + p.CB),
                     *reinterpret_cast<const uint2*>(rp + 2 * p.CB), t2);
        int q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int acc = __dp4a(static_cast<int>(t0[j]), static_cast<int>(wr[j][0]), 0);
          acc = __dp4a(static_cast<int>(t1[j]), static_cast<int>(wr[j][1]), acc);
          acc = __dp4a(static_cast<int>(t2[j]), static_cast<int>(wr[j][2]), acc);
          q[j] = requant_one(wrap_add(acc, bias[j]), scl[j], e);
        }
        const uint32_t lo = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
        const uint32_t hi = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
        *reinterpret_cast<uint2*>(yp) = make_uint2(lo, hi);
        yp += ystep;
        // slide the window: stride 1 keeps rows 1, 2; stride 2 keeps row 2 and transposes one more
        if constexpr (S == 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            t0[j] = t1[j];
            t1[j] = t2[j];
          }
          rp += pitch;
        } else {
          if (i + 1 < rows) {
#pragma unroll
            for (int j = 0; j < 8; ++j) t0[j] = t2[j];
            rp += pitch;
            dw_row_words(*reinterpret_cast<const uint2*>(rp), *reinterpret_cast<const uint2*>(rp + p.CB),
                         *reinterpret_cast<const uint2*>(rp + 2 * p.CB), t1);
            rp += pitch;
          }
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace b200q
