// Tensor-core route of the quantized-int32 drop-in conv (the reference's
// launch_{,block_}fprop_nhwc_qi32_{u8,s5}, src/cuda_kernels.cu:1336-1461).
//
// The reference computes y = sum over valid taps of (x - zx[n]) * (w - zw) on int32 codes that it
// stores as floats.  Centred U8 values reach +-255 and do not fit an 8-bit operand, so the raw
// codes go to the tensor core instead (U8 as unsigned, S5 as signed 8-bit operands) and the zero
// points come back as correction terms.  Let a_j be the raw input code of tap j, with the input's
// own zero point zx standing in for padding taps (a padding tap then contributes (zx - zx) = 0,
// exactly the reference's skip of invalid taps, src/cuda_kernels.cu:1196-1199), and b_j the raw
// weight code.  Over the T = R*S*Cg taps of a row:
//     sum (a_j - zx)(b_j - zw) = sum a_j b_j  - zw * sum a_j  - zx * sum b_j  + T * zx * zw
// All four terms are taken modulo 2^32, so the result equals the reference's wrapping int32
// accumulation bit for bit.
//
//   qi32_pack_kernel         one launch running both packs below (small problems; large ones
//                            launch qi32_pack_rows_kernel, then qi32_pack_filter_kernel):
//   qi32_pack_rows           float NHWC codes -> 8-bit im2col rows [G'][Mb][Kp] (G' = blocks x
//                            groups, Mb = pixels of one output block, Kp = T rounded up to 32) and
//                            the row term  T*zx*zw - zw*sum a_j  (int32, one per row);
//   qi32_pack_filter         float weights -> 8-bit rows [G'][Kg][Kp] and their sums  sum b_j;
//   tc_gemm_s8_kernel        C[G'][Mb][Kg] = A . B^T  (int32 out, unsigned or signed operands);
//   qi32_fixup_kernel        y[n,ho,wo,k] = C + rowterm - zx * colsum, scattered to NHWC.
// A regular conv (one block, one group) takes the correction in the GEMM's int32 epilogue instead
// (Epilogue::rowterm / rowzx, the column sums as its bias) and writes y directly; the fixup kernel
// then only runs the out-of-range fallback, returning at once when the flag is clear.
// Codes whose truncated value does not fit the 8-bit operand type (U8 outside [0, 255], S5
// outside [-128, 127]) set a device flag in the pack kernels (to the call's generation number, so
// the flag needs no clearing between calls: a stale or uninitialised value at worst runs the exact
// fallback); the fixup kernel then computes every
// output directly on CUDA cores (qi32_direct), so out-of-range inputs still give the reference's
// result, without a host round trip.
#pragma once
#include "simt.cuh"

namespace b200q {

// Direct quantized-int32 output element idx (the reference's loop nest, src/cpu_ref.cpp:36-112).
__device__ __noinline__ int32_t qi32_direct(const float* __restrict__ x, const float* __restrict__ w,
                                               const ConvGeom& g, size_t idx, const uint8_t* __restrict__ in_qp,
                                               int zf, int qp_stride, int qp_signed) {
  const int kk = static_cast<int>(idx % g.k);
  size_t pix = idx / g.k;
  const int wo = static_cast<int>(pix % g.wo);
  pix /= g.wo;
  const int ho = static_cast<int>(pix % g.ho);
  const int n = static_cast<int>(pix / g.ho);
  const int grp = kk / g.kg;
  const int by = ho / g.bho, bx = wo / g.bwo;
  const int zx = load_zp(in_qp, n, qp_stride, qp_signed);
  uint32_t acc = 0;
  for (int rr = 0; rr < g.r; ++rr) {
    const int hi = ho * g.stride_h - g.pad_h + rr * g.dil_h;
    if (hi < 0 || hi >= g.h) continue;
    for (int ss = 0; ss < g.s; ++ss) {
      const int wi = wo * g.stride_w - g.pad_w + ss * g.dil_w;
      if (wi < 0 || wi >= g.w) continue;
      const float* xp = x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + static_cast<size_t>(grp) * g.cg;
      const float* wp = w + ((((static_cast<size_t>(kk) * g.by + by) * g.bx + bx) * g.r + rr) * g.s + ss) * g.cg;
      for (int ci = 0; ci < g.cg; ++ci) {
        const int32_t xv = __float2int_rz(__ldg(xp + ci)) - zx;
        const int32_t wv = __float2int_rz(__ldg(wp + ci)) - zf;
        acc += static_cast<uint32_t>(xv) * static_cast<uint32_t>(wv);
      }
    }
  }
  return static_cast<int32_t>(acc);
}

// Truncated code of a float (static_cast<int32_t> semantics for in-range values) and whether it
// fits the operand type: unsigned [0, 255] or signed [-128, 127].
__device__ __forceinline__ int qi32_code(float f, int is_signed, bool& ok) {
  const int v = __float2int_rz(f);
  ok = is_signed ? (v >= -128 && v <= 127) : (v >= 0 && v <= 255);
  return v;
}

// Geometry of the packed problem, shared by the three kernels.
struct Qi32Pack {
  int T;       // taps per row: R * S * Cg
  int kp;      // packed row bytes: T rounded up to 32
  int mb;      // rows per block item: N * bho * bwo
  int gcount;  // G' = by * bx * groups
  int qp_stride, qp_signed;
  int gen;     // this call's generation number (nonzero): the out-of-range flag holds it when set
};

// One warp per packed row (gp, mb): gp = block * groups + group, mb = (image, row, column) inside
// the output block.  Each lane builds 4-byte words of the row; the row sum is reduced over the warp.
__device__ __forceinline__ void qi32_pack_rows(const float* __restrict__ x, uint32_t* __restrict__ a,
                                                             int32_t* __restrict__ rowterm, int32_t* __restrict__ rowzx,
                                                             ConvGeom g, Qi32Pack q,
                                                             const uint8_t* __restrict__ in_qp,
                                                             const uint8_t* __restrict__ f_qp, int* __restrict__ flag,
                                               int bid, int nblk) {
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(q.gcount) * q.mb;
  const long long warp0 = (static_cast<long long>(bid) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(nblk) * blockDim.x) >> 5;
  const int zf = load_zp(f_qp, 0, q.qp_stride, q.qp_signed);
  const int words = q.kp >> 2;
  const int sc = g.s * g.cg;
  bool bad = false;
  // Channels of a group in multiples of 4 with a 16-byte aligned x: every word is 4 consecutive
  // channels of one tap, read with one 16-byte load (consecutive lanes, consecutive 16 bytes).
  const bool v4 = (g.cg & 3) == 0 && (g.c & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const uint32_t bias8 = q.qp_signed ? 128u : 0u;
  const bool one_gp = q.gcount == 1;  // a regular conv: row = pixel, no block / group decode
  for (long long row = warp0; row < rows; row += nwarps) {
    int gp = 0, rem;
    if (one_gp) {
      rem = static_cast<int>(row);
    } else {
      gp = static_cast<int>(row / q.mb);
      rem = static_cast<int>(row - static_cast<long long>(gp) * q.mb);
    }
    const int grp = one_gp ? 0 : gp % g.groups, blk = one_gp ? 0 : gp / g.groups;
    const int byi = one_gp ? 0 : blk / g.bx, bxi = blk - byi * g.bx;
    const int owb = rem % g.bwo;
    rem /= g.bwo;
    const int ohb = rem % g.bho;
    const int n = rem / g.bho;
    const int ho = byi * g.bho + ohb, wo = bxi * g.bwo + owb;
    const int zx = load_zp(in_qp, n, q.qp_stride, q.qp_signed);
    const int h0 = ho * g.stride_h - g.pad_h, w0 = wo * g.stride_w - g.pad_w;
    const float* xn = x + static_cast<size_t>(n) * g.h * g.w * g.c + static_cast<size_t>(grp) * g.cg;
    uint32_t* arow = a + static_cast<size_t>(row) * words;
    uint32_t sum = 0;
    if (v4) {
      // The lane's tap position (rr, ss, ci) of word wd advances by 128 taps per step (32 lanes x 4
      // channels); divisions run only when ci leaves the group's channels (rarely for wide groups).
      int j0 = lane * 4;
      int rr = j0 / sc;
      int ss = (j0 - rr * sc) / g.cg;
      int ci = j0 - rr * sc - ss * g.cg;
#pragma unroll 4
      for (int wd = lane; wd < words; wd += 32, j0 += 128) {
        uint32_t word = 0;
        if (j0 < q.T) {
          const int hi = h0 + rr * g.dil_h, wi = w0 + ss * g.dil_w;
          int v0 = zx, v1 = zx, v2 = zx, v3 = zx;
          if (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w) {
            const float4 f = __ldg(reinterpret_cast<const float4*>(xn + (static_cast<size_t>(hi) * g.w + wi) * g.c + ci));
            v0 = __float2int_rz(f.x);
            v1 = __float2int_rz(f.y);
            v2 = __float2int_rz(f.z);
            v3 = __float2int_rz(f.w);
            // a code fits iff (v + bias8) lies in [0, 255] (bias8 = 128 signed, 0 unsigned): one test
            // of the OR of the four shifted codes against the bits above the low byte
            const uint32_t any = (static_cast<uint32_t>(v0) + bias8) | (static_cast<uint32_t>(v1) + bias8) |
                                 (static_cast<uint32_t>(v2) + bias8) | (static_cast<uint32_t>(v3) + bias8);
            bad |= (any & ~0xFFu) != 0;
          }
          sum += static_cast<uint32_t>(v0) + static_cast<uint32_t>(v1) + static_cast<uint32_t>(v2) +
                 static_cast<uint32_t>(v3);
          word = __byte_perm(__byte_perm(v0, v1, 0x0040), __byte_perm(v2, v3, 0x0040), 0x5410);
          ci += 128;
          if (ci >= g.cg) {
            const int carry = ci / g.cg;
            ci -= carry * g.cg;
            ss += carry;
            if (ss >= g.s) {
              rr += ss / g.s;
              ss %= g.s;
            }
          }
        }
        arow[wd] = word;
      }
    } else
    for (int wd = lane; wd < words; wd += 32) {
      uint32_t word = 0;
      const int j0 = wd * 4;
      if (j0 < q.T) {
        int rr = j0 / sc;
        int t = j0 - rr * sc;
        int ss = t / g.cg;
        int ci = t - ss * g.cg;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          int v = 0;
          if (j0 + b < q.T) {
            const int hi = h0 + rr * g.dil_h, wi = w0 + ss * g.dil_w;
            if (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w) {
              bool ok;
              v = qi32_code(__ldg(xn + (static_cast<size_t>(hi) * g.w + wi) * g.c + ci), q.qp_signed, ok);
              bad |= !ok;
            } else {
              v = zx;
            }
            sum += static_cast<uint32_t>(v);
            if (++ci == g.cg) {
              ci = 0;
              if (++ss == g.s) {
                ss = 0;
                ++rr;
              }
            }
          }
          word |= (static_cast<uint32_t>(v) & 0xFFu) << (8 * b);
        }
      }
      arow[wd] = word;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) {
      rowterm[row] = static_cast<int32_t>(static_cast<uint32_t>(q.T) * static_cast<uint32_t>(zx) * static_cast<uint32_t>(zf) -
                                          static_cast<uint32_t>(zf) * sum);
      rowzx[row] = zx;
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) *reinterpret_cast<volatile int*>(flag) = q.gen;
}

// One warp per packed filter row (gp, kg): the weights of output channel grp * Kg + kg for output
// block (byi, bxi), from [K][By][Bx][R][S][Cg] float codes.  colsum = sum of the row's codes.
__device__ __forceinline__ void qi32_pack_filter(const float* __restrict__ w, uint32_t* __restrict__ b,
                                                               int32_t* __restrict__ colsum, ConvGeom g, Qi32Pack q,
                                                               int* __restrict__ flag, int bid, int nblk) {
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(q.gcount) * g.kg;
  const long long warp0 = (static_cast<long long>(bid) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(nblk) * blockDim.x) >> 5;
  const int words = q.kp >> 2;
  bool bad = false;
  for (long long row = warp0; row < rows; row += nwarps) {
    const int gp = static_cast<int>(row / g.kg);
    const int kg = static_cast<int>(row - static_cast<long long>(gp) * g.kg);
    const int grp = gp % g.groups, blk = gp / g.groups;
    const int kk = grp * g.kg + kg;
    // filter slice of (kk, block): blocks are [By][Bx] = blk in row-major order
    const float* wr = w + (static_cast<size_t>(kk) * g.by * g.bx + blk) * q.T;
    uint32_t* brow = b + static_cast<size_t>(row) * words;
    uint32_t sum = 0;
    for (int wd = lane; wd < words; wd += 32) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = wd * 4 + i;
        if (j < q.T) {
          bool ok;
          const int v = qi32_code(__ldg(wr + j), q.qp_signed, ok);
          bad |= !ok;
          sum += static_cast<uint32_t>(v);
          word |= (static_cast<uint32_t>(v) & 0xFFu) << (8 * i);
        }
      }
      brow[wd] = word;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    if (lane == 0) colsum[row] = static_cast<int32_t>(sum);
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) *reinterpret_cast<volatile int*>(flag) = q.gen;
}

// Both packs in one launch (a call of the drop-in is short and launch-latency-bound at small sizes):
// blocks [0, row_blocks) pack the activation rows, the rest (if any) pack the filter rows.
__global__ void __launch_bounds__(256) qi32_pack_kernel(const float* __restrict__ x, uint32_t* __restrict__ a,
                                                        int32_t* __restrict__ rowterm, int32_t* __restrict__ rowzx,
                                                        const float* __restrict__ w, uint32_t* __restrict__ b,
                                                        int32_t* __restrict__ colsum, ConvGeom g, Qi32Pack q,
                                                        const uint8_t* __restrict__ in_qp,
                                                        const uint8_t* __restrict__ f_qp, int* __restrict__ flag,
                                                        int row_blocks) {
  const int bid = static_cast<int>(blockIdx.x);
  if (bid < row_blocks)
    qi32_pack_rows(x, a, rowterm, rowzx, g, q, in_qp, f_qp, flag, bid, row_blocks);
  else
    qi32_pack_filter(w, b, colsum, g, q, flag, bid - row_blocks, static_cast<int>(gridDim.x) - row_blocks);
}

// The two packs as separate kernels (large problems; each kernel keeps its own register budget).
__global__ void __launch_bounds__(256) qi32_pack_rows_kernel(const float* __restrict__ x, uint32_t* __restrict__ a,
                                                             int32_t* __restrict__ rowterm, int32_t* __restrict__ rowzx,
                                                             ConvGeom g, Qi32Pack q, const uint8_t* __restrict__ in_qp,
                                                             const uint8_t* __restrict__ f_qp, int* __restrict__ flag) {
  qi32_pack_rows(x, a, rowterm, rowzx, g, q, in_qp, f_qp, flag, static_cast<int>(blockIdx.x),
                 static_cast<int>(gridDim.x));
}

__global__ void __launch_bounds__(256) qi32_pack_filter_kernel(const float* __restrict__ w, uint32_t* __restrict__ b,
                                                               int32_t* __restrict__ colsum, ConvGeom g, Qi32Pack q,
                                                               int* __restrict__ flag) {
  qi32_pack_filter(w, b, colsum, g, q, flag, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x));
}

// Output element (n, ho, wo, k) from the GEMM accumulators C[gp][mb][kg] (src may alias y when
// G' == 1: then the mapping is the identity and each thread reads its own element before writing
// it).  With the flag set (a code did not fit its 8-bit type) every output is computed directly.
// Four consecutive output channels per thread when Kg % 4 == 0 (16-byte loads and stores).
template <int V>
__global__ void __launch_bounds__(256) qi32_fixup_kernel(const int32_t* src, int32_t* y,
                                                         const int32_t* __restrict__ rowterm,
                                                         const int32_t* __restrict__ colsum, ConvGeom g, Qi32Pack q,
                                                         const uint8_t* __restrict__ in_qp,
                                                         const uint8_t* __restrict__ f_qp, const int* __restrict__ flag,
                                                         const float* __restrict__ x, const float* __restrict__ w,
                                                         int fused) {
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  const size_t items = total / V;
  const bool direct = *reinterpret_cast<const volatile int*>(flag) == q.gen;
  // fused: the GEMM epilogue already applied the correction; only the out-of-range fallback is left
  if (fused && !direct) return;
  const int zf = load_zp(f_qp, 0, q.qp_stride, q.qp_signed);
  for (size_t it = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t idx = it * V;
    if (direct) {
#pragma unroll
      for (int v = 0; v < V; ++v) y[idx + v] = qi32_direct(x, w, g, idx + v, in_qp, zf, q.qp_stride, q.qp_signed);
      continue;
    }
    const int kk = static_cast<int>(idx % g.k);
    size_t pix = idx / g.k;
    const int wo = static_cast<int>(pix % g.wo);
    pix /= g.wo;
    const int ho = static_cast<int>(pix % g.ho);
    const int n = static_cast<int>(pix / g.ho);
    const int grp = kk / g.kg, kg = kk - grp * g.kg;
    const int byi = ho / g.bho, bxi = wo / g.bwo;
    const int gp = (byi * g.bx + bxi) * g.groups + grp;
    const long long mb = (static_cast<long long>(n) * g.bho + (ho - byi * g.bho)) * g.bwo + (wo - bxi * g.bwo);
    const long long prow = static_cast<long long>(gp) * q.mb + mb;
    const uint32_t zx = static_cast<uint32_t>(load_zp(in_qp, n, q.qp_stride, q.qp_signed));
    const uint32_t rt = static_cast<uint32_t>(__ldg(rowterm + prow));
    const int32_t* cs = colsum + static_cast<size_t>(gp) * g.kg + kg;
    const int32_t* sp = src + static_cast<size_t>(prow) * g.kg + kg;
    if constexpr (V == 4) {
      const int4 c4 = *reinterpret_cast<const int4*>(sp);
      const int4 s4 = *reinterpret_cast<const int4*>(cs);
      int4 o;
      o.x = static_cast<int32_t>(static_cast<uint32_t>(c4.x) + rt - zx * static_cast<uint32_t>(s4.x));
      o.y = static_cast<int32_t>(static_cast<uint32_t>(c4.y) + rt - zx * static_cast<uint32_t>(s4.y));
      o.z = static_cast<int32_t>(static_cast<uint32_t>(c4.z) + rt - zx * static_cast<uint32_t>(s4.z));
      o.w = static_cast<int32_t>(static_cast<uint32_t>(c4.w) + rt - zx * static_cast<uint32_t>(s4.w));
      *reinterpret_cast<int4*>(y + idx) = o;
    } else {
      y[idx] = static_cast<int32_t>(static_cast<uint32_t>(*sp) + rt - zx * static_cast<uint32_t>(__ldg(cs)));
    }
  }
}

}  // namespace b200q
