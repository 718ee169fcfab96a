// CUDA-core kernels of the b200q library (exact integer arithmetic):
//  - quantized-int32 conv on float codes with zero points (the drop-in for the reference's
//    launch_{,block_}fprop_nhwc_qi32_*): one fused gather/centre/MAC kernel for all groups and
//    output blocks, no workspace, no memset, every output element written once;
//  - int8 direct conv with dp4a for shapes the tensor-core path does not take (C % 32 != 0,
//    grouped, tiny tensors), with the fused requantization epilogue;
//  - depthwise int8 conv (groups == C == K), 128-bit loads, weights staged in shared memory;
//  - tiled batched GEMM for int32 (wrap-around) and int8 inputs;
//  - counter-based synthetic data generators.
#pragma once
#include "common.cuh"

namespace b200q {

struct ConvGeom {
  int n, h, w, c, r, s, k, ho, wo;
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w;
  int groups, cg, kg;
  int by, bx, bho, bwo;  // block grid (1,1 for a regular conv) and block extents
};

// Zero point of qparams element i: byte 0 of a struct of `stride` bytes, unsigned (U8) or signed (S5).
__device__ __forceinline__ int load_zp(const uint8_t* qp, int i, int stride, int is_signed) {
  const uint8_t b = qp[static_cast<size_t>(i) * stride];
  return is_signed ? static_cast<int>(static_cast<int8_t>(b)) : static_cast<int>(b);
}

// y[n,ho,wo,kk] = sum_{valid r,s} sum_ci (int(x) - zp_in[n]) * (int(w) - zp_f); int32 wrap.
// Follows src/cpu_ref.cpp:36-112 (one thread per output element).
__global__ void qi32_conv_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                 int32_t* __restrict__ y, ConvGeom g, const uint8_t* __restrict__ in_qp,
                                 const uint8_t* __restrict__ f_qp, int qp_stride, int qp_signed) {
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  const int zf = load_zp(f_qp, 0, qp_stride, qp_signed);
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
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
    y[idx] = static_cast<int32_t>(acc);
  }
}

// int8 direct conv, one thread per output element, dp4a over 4-channel words when aligned.
__global__ void conv_s8_generic_kernel(const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                       void* __restrict__ y, ConvGeom g, Epilogue e, int use_dp4a) {
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int kk = static_cast<int>(idx % g.k);
    size_t pix = idx / g.k;
    const int wo = static_cast<int>(pix % g.wo);
    pix /= g.wo;
    const int ho = static_cast<int>(pix % g.ho);
    const int n = static_cast<int>(pix / g.ho);
    const int grp = kk / g.kg;
    int32_t acc = 0;
    for (int rr = 0; rr < g.r; ++rr) {
      const int hi = ho * g.stride_h - g.pad_h + rr * g.dil_h;
      if (hi < 0 || hi >= g.h) continue;
      for (int ss = 0; ss < g.s; ++ss) {
        const int wi = wo * g.stride_w - g.pad_w + ss * g.dil_w;
        if (wi < 0 || wi >= g.w) continue;
        const int8_t* xp = x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + static_cast<size_t>(grp) * g.cg;
        const int8_t* wp = w + ((static_cast<size_t>(kk) * g.r + rr) * g.s + ss) * g.cg;
        if (use_dp4a) {
          const int* xw = reinterpret_cast<const int*>(xp);
          const int* ww = reinterpret_cast<const int*>(wp);
          for (int q = 0; q < (g.cg >> 2); ++q) acc = __dp4a(__ldg(xw + q), __ldg(ww + q), acc);
        } else {
          for (int ci = 0; ci < g.cg; ++ci)
            acc += static_cast<int32_t>(__ldg(xp + ci)) * static_cast<int32_t>(__ldg(wp + ci));
        }
      }
    }
    epilogue_store(e, y, idx, acc, kk);
  }
}

// Depthwise int8 conv, 3x3 taps (groups == C == K, C % 8 == 0).  A thread owns 8 channels
// (cgroup) for a strided set of output pixels.  Per pixel it loads the 8 channels of each tap
// (one 8-byte load; consecutive threads take consecutive channel groups of the same pixel, so a
// warp's loads are contiguous), byte-transposes the words of taps 0-3 and 4-7 with 8 prmt per
// 4x4 block so that one word holds one channel's 4 taps, and accumulates with dp4a against the
// channel's packed weights (4 MACs per instruction).  Tap 8 uses a weight pre-shifted into the
// channel's byte lane, so a dp4a with the raw activation word picks exactly that channel.
constexpr int kDwMaxTaps = 9;

// 4x4 byte transpose: in[i] byte j -> out[j] byte i.
__device__ __forceinline__ void transpose4x4_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t& o0,
                                                   uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(c, d, 0x5140);
  const uint32_t t2 = __byte_perm(a, b, 0x7362), t3 = __byte_perm(c, d, 0x7362);
  o0 = __byte_perm(t0, t1, 0x5410);
  o1 = __byte_perm(t0, t1, 0x7632);
  o2 = __byte_perm(t2, t3, 0x5410);
  o3 = __byte_perm(t2, t3, 0x7632);
}

template <int KIND>
__global__ void __launch_bounds__(256) dw_conv_s8_kernel(const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                                         void* __restrict__ y, ConvGeom g, Epilogue e) {
  const int groups8 = g.c >> 3;
  const int lanes_per_block = blockDim.x / groups8;  // pixels handled by one block at a time
  const int cg = threadIdx.x % groups8;
  const int pl = threadIdx.x / groups8;
  if (pl >= lanes_per_block) return;
  const int c0 = cg * 8;
  // packed weights: wq[j][0] = taps 0-3 of channel c0+j, wq[j][1] = taps 4-7; w8[j] = tap 8 shifted
  uint32_t wq[8][2], w8[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int8_t* wp = w + static_cast<size_t>(c0 + j) * 9;
    uint32_t v[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) v[t] = static_cast<uint8_t>(__ldg(wp + t));
    wq[j][0] = v[0] | (v[1] << 8) | (v[2] << 16) | (v[3] << 24);
    wq[j][1] = v[4] | (v[5] << 8) | (v[6] << 16) | (v[7] << 24);
    w8[j] = v[8] << (8 * (j & 3));
  }
  int32_t bsum[8];
  float sc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bsum[j] = e.bias ? __ldg(e.bias + c0 + j) : 0;
    sc[j] = e.scale ? __ldg(e.scale + c0 + j) : 0.0f;
  }
  const int npix = g.n * g.ho * g.wo;  // < 2^31 (checked by the caller)
  const int row_pitch = g.w * g.c;
  for (int pix = blockIdx.x * lanes_per_block + pl; pix < npix; pix += gridDim.x * lanes_per_block) {
    const int wo = pix % g.wo;
    const int t2 = pix / g.wo;
    const int ho = t2 % g.ho;
    const int n = t2 / g.ho;
    const int h0 = ho * g.stride_h - g.pad_h, w0 = wo * g.stride_w - g.pad_w;
    const int8_t* base = x + (static_cast<size_t>(n) * g.h * g.w) * g.c + c0;
    uint32_t xl[9], xh[9];  // channels 0-3 / 4-7 of each tap (0 at padding)
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const int hi = h0 + (t / 3) * g.dil_h, wi = w0 + (t % 3) * g.dil_w;
      uint2 v = make_uint2(0u, 0u);
      if (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w)
        v = __ldg(reinterpret_cast<const uint2*>(base + hi * row_pitch + wi * g.c));
      xl[t] = v.x;
      xh[t] = v.y;
    }
    int acc[8];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t* xs = half ? xh : xl;
      uint32_t c[4], d[4];
      transpose4x4_bytes(xs[0], xs[1], xs[2], xs[3], c[0], c[1], c[2], c[3]);
      transpose4x4_bytes(xs[4], xs[5], xs[6], xs[7], d[0], d[1], d[2], d[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ch = half * 4 + j;
        int a = __dp4a(static_cast<int>(c[j]), static_cast<int>(wq[ch][0]), 0);
        a = __dp4a(static_cast<int>(d[j]), static_cast<int>(wq[ch][1]), a);
        acc[ch] = __dp4a(static_cast<int>(xs[8]), static_cast<int>(w8[ch]), a);
      }
    }
    const size_t o = static_cast<size_t>(pix) * g.c + c0;
    if constexpr (KIND == kOutS8) {
      int q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = requant_one(wrap_add(acc[j], bsum[j]), sc[j], e);
      const uint32_t lo = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
      const uint32_t hi = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
      *reinterpret_cast<uint2*>(static_cast<int8_t*>(y) + o) = make_uint2(lo, hi);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) epilogue_store(e, y, o + j, acc[j], c0 + j);
    }
  }
}

// Tiled batched GEMM on CUDA cores: 64x64 output tile per 256 threads, 4x4 per thread, BK=16.
// C_b = op(A_b) @ op(B_b) with bmm.h:9-29 layouts; products and sums in uint32 (wrap-around),
// which is bmm.cu:218-229's int32 arithmetic without signed-overflow UB.
template <typename T>
__global__ void __launch_bounds__(256) bmm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                       void* __restrict__ C, int M, int N, int K,
                                                       int ta, int tb, Epilogue e, const int* run_if, int run_gen,
                                                       int batch) {
  // run_if: when given, the block does nothing unless *run_if == run_gen (the int32 bmm's fallback
  // after its tensor-core route found an operand outside the 8-bit range in call run_gen).
  // The block walks 64 x 64 output tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... of all batches.
  if (run_if && *reinterpret_cast<const volatile int*>(run_if) != run_gen) return;
  __shared__ int32_t As[16][64 + 1];
  __shared__ int32_t Bs[16][64 + 1];
  const int tn = (N + 63) / 64, tm = (M + 63) / 64;
  const long long tiles = static_cast<long long>(tn) * tm * batch;
  for (long long t = blockIdx.x; t < tiles; t += gridDim.x) {
  const int b = static_cast<int>(t / (static_cast<long long>(tn) * tm));
  const int rem = static_cast<int>(t - static_cast<long long>(b) * tn * tm);
  const int m0 = (rem / tn) * 64, n0 = (rem % tn) * 64;
  const T* Ab = A + static_cast<size_t>(b) * M * K;
  const T* Bb = B + static_cast<size_t>(b) * K * N;
  const int tid = threadIdx.x;
  const int tr = (tid >> 4) * 4, tc = (tid & 15) * 4;
  uint32_t acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = tid; i < 1024; i += 256) {
      int mm, kk;
      if (ta) { mm = i & 63; kk = i >> 6; } else { kk = i & 15; mm = i >> 4; }
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? static_cast<int32_t>(ta ? Ab[static_cast<size_t>(gk) * M + gm]
                                                                 : Ab[static_cast<size_t>(gm) * K + gk])
                                      : 0;
      int nn, k2;
      if (tb) { k2 = i & 15; nn = i >> 4; } else { nn = i & 63; k2 = i >> 6; }
      const int gn = n0 + nn, gk2 = k0 + k2;
      Bs[k2][nn] = (gn < N && gk2 < K) ? static_cast<int32_t>(tb ? Bb[static_cast<size_t>(gn) * K + gk2]
                                                                  : Bb[static_cast<size_t>(gk2) * N + gn])
                                       : 0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      uint32_t av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = static_cast<uint32_t>(As[kk][tr + i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = static_cast<uint32_t>(Bs[kk][tc + j]);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tr + i;
    if (m >= M) continue;
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tc + j;
      if (n < N)
        epilogue_store(e, C, static_cast<size_t>(b) * M * N + static_cast<size_t>(m) * N + n,
                       static_cast<int32_t>(acc[i][j]), n);
    }
  }
  }
}

// int32 operands -> int8 copies for the tensor-core route of the int32 bmm (bmm.cu:298-322 computes
// on arbitrary int32 values).  One launch converts both operands: unit u < na / 16 is 16 values of
// A, the rest are 16 values of B (na, nb multiples of 16; sources 16-byte, destinations 16-byte
// aligned); each thread has its four 16-byte loads in flight before it stores.  A value outside
// [-128, 127] sets *flag to the call's generation number gen; the CUDA-core kernel then recomputes C
// from the int32 operands, so the
// result stays the reference's for every input without a host round trip.
__device__ __forceinline__ bool s8_out_of_range(const int4& v) {
  return static_cast<uint32_t>(v.x + 128) > 255u || static_cast<uint32_t>(v.y + 128) > 255u ||
         static_cast<uint32_t>(v.z + 128) > 255u || static_cast<uint32_t>(v.w + 128) > 255u;
}
__device__ __forceinline__ uint32_t pack4_s8_trunc(const int4& v) {
  return __byte_perm(__byte_perm(v.x, v.y, 0x0040), __byte_perm(v.z, v.w, 0x0040), 0x5410);
}
__global__ void __launch_bounds__(256) i32_to_s8_kernel(const int32_t* __restrict__ a, int8_t* __restrict__ a8,
                                                        size_t na, const int32_t* __restrict__ b,
                                                        int8_t* __restrict__ b8, size_t nb, int* __restrict__ flag,
                                                        int gen) {
  const size_t ua = na / 16, units = ua + nb / 16;
  const size_t step = static_cast<size_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  for (size_t u = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < units; u += step) {
    const bool in_a = u < ua;
    const size_t k = in_a ? u : u - ua;
    const int4* src = reinterpret_cast<const int4*>(in_a ? a : b) + 4 * k;
    const int4 v0 = __ldg(src), v1 = __ldg(src + 1), v2 = __ldg(src + 2), v3 = __ldg(src + 3);
    bad |= s8_out_of_range(v0) || s8_out_of_range(v1) || s8_out_of_range(v2) || s8_out_of_range(v3);
    reinterpret_cast<uint4*>(in_a ? a8 : b8)[k] =
        make_uint4(pack4_s8_trunc(v0), pack4_s8_trunc(v1), pack4_s8_trunc(v2), pack4_s8_trunc(v3));
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) *reinterpret_cast<volatile int*>(flag) = gen;
}

// ------------------------------------------------------------------ generators
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t draw64(uint64_t key, uint64_t i) {
  return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
}

__global__ void fill_s8_uniform_kernel(int8_t* out, size_t count, uint64_t key, int lo, uint64_t span) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = static_cast<int8_t>(lo + static_cast<int>(((draw64(key, i) >> 32) * span) >> 32));
}
__global__ void fill_i32_uniform_kernel(int32_t* out, size_t count, uint64_t key, long long lo, uint64_t span) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = static_cast<int32_t>(lo + static_cast<long long>(((draw64(key, i) >> 32) * span) >> 32));
}
__global__ void fill_s8_table_kernel(int8_t* out, size_t count, uint64_t key, const int8_t* __restrict__ table) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __ldg(table + (draw64(key, i) >> 48));
}

}  // namespace b200q

namespace b200q {

// Low-channel convolutions (C % 16 != 0, e.g. the C = 3 stems) on the tensor cores: the
// activation rows are gathered into an im2col matrix a[m][kp] with kp = round_up(R*S*C, 32),
// columns ordered (r, s, c) like the KRSC weights, zero at padding taps and past R*S*C.
// A block builds `rows` consecutive matrix rows in shared memory (one thread per (row, tap)
// copies the tap's C channels) and then writes the tile -- contiguous in the matrix -- with
// 16-byte stores.
__global__ void __launch_bounds__(256) im2col_pack_s8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ a,
                                                             ConvGeom g, int kp, long long total_rows, int rows) {
  extern __shared__ __align__(16) int8_t tile[];
  const int rsc = g.r * g.s * g.c;
  for (long long m0 = static_cast<long long>(blockIdx.x) * rows; m0 < total_rows;
       m0 += static_cast<long long>(gridDim.x) * rows) {
    const int nrows = static_cast<int>(min(static_cast<long long>(rows), total_rows - m0));
    // zero the padding columns [rsc, kp) of every row
    const int padw = kp - rsc;
    if (padw > 0)
      for (int i = threadIdx.x; i < nrows * padw; i += blockDim.x) tile[(i / padw) * kp + rsc + i % padw] = 0;
    // one work item = (row, filter row rr): S taps x C channels, coordinates decoded once
    for (int it = threadIdx.x; it < nrows * g.r; it += blockDim.x) {
      const int lr = it / g.r;
      const int rr = it - lr * g.r;
      const int m = static_cast<int>(m0) + lr;  // < 2^31 (checked by the caller)
      const int wo = m % g.wo;
      const int t = m / g.wo;
      const int ho = t % g.ho;
      const int n = t / g.ho;
      const int hi = ho * g.stride_h - g.pad_h + rr * g.dil_h;
      int8_t* dst = tile + lr * kp + rr * g.s * g.c;
      if (hi < 0 || hi >= g.h) {
        for (int i = 0; i < g.s * g.c; ++i) dst[i] = 0;
        continue;
      }
      const int8_t* row = x + (static_cast<size_t>(n) * g.h + hi) * g.w * g.c;
      for (int ss = 0; ss < g.s; ++ss) {
        const int wi = wo * g.stride_w - g.pad_w + ss * g.dil_w;
        if (wi >= 0 && wi < g.w) {
          const int8_t* src = row + static_cast<size_t>(wi) * g.c;
          for (int c = 0; c < g.c; ++c) dst[ss * g.c + c] = __ldg(src + c);
        } else {
          for (int c = 0; c < g.c; ++c) dst[ss * g.c + c] = 0;
        }
      }
    }
    __syncthreads();
    int4* out = reinterpret_cast<int4*>(a + m0 * kp);
    const int4* src = reinterpret_cast<const int4*>(tile);
    for (int i = threadIdx.x; i < nrows * kp / 16; i += blockDim.x) out[i] = src[i];
    __syncthreads();
  }
}

// Depthwise 3x3 with dilation 1, PX horizontally adjacent output pixels per thread (stride_w =
// SW): the 3 x ((PX - 1) * SW + 3) input words the pixels share are loaded once (stride 1, PX = 8:
// 30 loads for 8 pixels instead of 72), unconditionally when the window is inside the image.  The
// per-pixel arithmetic is the one of dw_conv_s8_kernel.
template <int KIND, int SW, int PX>
__global__ void __launch_bounds__(256) dw_conv_s8_px_kernel(const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                                            void* __restrict__ y, ConvGeom g, Epilogue e) {
  constexpr int NC = (PX - 1) * SW + 3;
  const int groups8 = g.c >> 3;
  const int lanes_per_block = blockDim.x / groups8;
  const int cg = threadIdx.x % groups8;
  const int pl = threadIdx.x / groups8;
  if (pl >= lanes_per_block) return;
  const int c0 = cg * 8;
  uint32_t wq[8][2], w8[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int8_t* wp = w + static_cast<size_t>(c0 + j) * 9;
    uint32_t v[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) v[t] = static_cast<uint8_t>(__ldg(wp + t));
    wq[j][0] = v[0] | (v[1] << 8) | (v[2] << 16) | (v[3] << 24);
    wq[j][1] = v[4] | (v[5] << 8) | (v[6] << 16) | (v[7] << 24);
    w8[j] = v[8] << (8 * (j & 3));
  }
  int32_t bsum[8];
  float sc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bsum[j] = e.bias ? __ldg(e.bias + c0 + j) : 0;
    sc[j] = e.scale ? __ldg(e.scale + c0 + j) : 0.0f;
  }
  const int wgroups = (g.wo + PX - 1) / PX;
  const int nitems = g.n * g.ho * wgroups;  // < 2^31 (checked by the caller)
  const int row_pitch = g.w * g.c;
  for (int it = blockIdx.x * lanes_per_block + pl; it < nitems; it += gridDim.x * lanes_per_block) {
    const int wgi = it % wgroups;
    const int t2 = it / wgroups;
    const int ho = t2 % g.ho;
    const int n = t2 / g.ho;
    const int wo0 = wgi * PX;
    const int h0 = ho * g.stride_h - g.pad_h, w0 = wo0 * SW - g.pad_w;
    const int8_t* base = x + (static_cast<size_t>(n) * g.h * g.w) * g.c + c0;
    uint2 v[3][NC];
    if (h0 >= 0 && h0 + 2 < g.h && w0 >= 0 && w0 + NC - 1 < g.w) {
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int cc = 0; cc < NC; ++cc)
          v[r][cc] = __ldg(reinterpret_cast<const uint2*>(base + (h0 + r) * row_pitch + (w0 + cc) * g.c));
    } else {
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int cc = 0; cc < NC; ++cc) {
          const int hi = h0 + r, wi = w0 + cc;
          v[r][cc] = (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w)
                         ? __ldg(reinterpret_cast<const uint2*>(base + hi * row_pitch + wi * g.c))
                         : make_uint2(0u, 0u);
        }
    }
#pragma unroll
    for (int p = 0; p < PX; ++p) {
      if (wo0 + p >= g.wo) break;
      uint32_t xl[9], xh[9];
#pragma unroll
      for (int t = 0; t < 9; ++t) {
        xl[t] = v[t / 3][p * SW + t % 3].x;
        xh[t] = v[t / 3][p * SW + t % 3].y;
      }
      int acc[8];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t* xs = half ? xh : xl;
        uint32_t c[4], d[4];
        transpose4x4_bytes(xs[0], xs[1], xs[2], xs[3], c[0], c[1], c[2], c[3]);
        transpose4x4_bytes(xs[4], xs[5], xs[6], xs[7], d[0], d[1], d[2], d[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = half * 4 + j;
          int a = __dp4a(static_cast<int>(c[j]), static_cast<int>(wq[ch][0]), 0);
          a = __dp4a(static_cast<int>(d[j]), static_cast<int>(wq[ch][1]), a);
          acc[ch] = __dp4a(static_cast<int>(xs[8]), static_cast<int>(w8[ch]), a);
        }
      }
      const size_t o = (static_cast<size_t>(t2) * g.wo + wo0 + p) * g.c + c0;
      if constexpr (KIND == kOutS8) {
        int q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = requant_one(wrap_add(acc[j], bsum[j]), sc[j], e);
        const uint32_t lo = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
        const uint32_t hi = __byte_perm(__byte_perm(q[4], q[5], 0x0040), __byte_perm(q[6], q[7], 0x0040), 0x5410);
        *reinterpret_cast<uint2*>(static_cast<int8_t*>(y) + o) = make_uint2(lo, hi);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) epilogue_store(e, y, o + j, acc[j], c0 + j);
      }
    }
  }
}

// Max pool, NHWC int8: one thread = one output pixel x 16 channels (C % 16 == 0) using 4-lane
// signed byte max, or one output element otherwise.  Padded positions take no part (a window that
// lies entirely in the padding gives -128).
__global__ void maxpool_s8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ y, ConvGeom g) {
  const bool vec = g.c % 16 == 0;
  const int cv = vec ? g.c / 16 : g.c;
  const long long total = static_cast<long long>(g.n) * g.ho * g.wo * cv;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int cc = static_cast<int>(idx % cv);
    const long long pix = idx / cv;
    const int wo = static_cast<int>(pix % g.wo);
    const long long t = pix / g.wo;
    const int ho = static_cast<int>(t % g.ho);
    const int n = static_cast<int>(t / g.ho);
    const int8_t* base = x + static_cast<size_t>(n) * g.h * g.w * g.c;
    if (vec) {
      uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
      for (int i = 0; i < g.r; ++i) {
        const int hi = ho * g.stride_h - g.pad_h + i;
        if (hi < 0 || hi >= g.h) continue;
        for (int j = 0; j < g.s; ++j) {
          const int wi = wo * g.stride_w - g.pad_w + j;
          if (wi < 0 || wi >= g.w) continue;
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (static_cast<size_t>(hi) * g.w + wi) * g.c) + cc);
          m.x = __vmaxs4(m.x, v.x); m.y = __vmaxs4(m.y, v.y); m.z = __vmaxs4(m.z, v.z); m.w = __vmaxs4(m.w, v.w);
        }
      }
      reinterpret_cast<uint4*>(y + pix * g.c)[cc] = m;
    } else {
      int m = -128;
      for (int i = 0; i < g.r; ++i) {
        const int hi = ho * g.stride_h - g.pad_h + i;
        if (hi < 0 || hi >= g.h) continue;
        for (int j = 0; j < g.s; ++j) {
          const int wi = wo * g.stride_w - g.pad_w + j;
          if (wi < 0 || wi >= g.w) continue;
          m = max(m, static_cast<int>(base[(static_cast<size_t>(hi) * g.w + wi) * g.c + cc]));
        }
      }
      y[pix * g.c + cc] = static_cast<int8_t>(m);
    }
  }
}

// Global average pool, NHWC int8 -> [n][c]: one warp per (image, 32-channel group); lanes stride
// over the pixels with exact int32 sums, then q = clamp(rint_sat(sum / (h*w)), -128, 127) with one
// IEEE division.
__global__ void global_avgpool_s8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ y, int n, int hw,
                                         int c) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cgroups = (c + 31) / 32;
  const long long items = static_cast<long long>(n) * cgroups;
  const float cnt = static_cast<float>(hw);
  for (long long it = blockIdx.x * static_cast<long long>(warps) + (threadIdx.x >> 5); it < items;
       it += static_cast<long long>(gridDim.x) * warps) {
    const int b = static_cast<int>(it / cgroups);
    const int ch = static_cast<int>(it % cgroups) * 32 + lane;
    if (ch >= c) continue;
    const int8_t* p = x + static_cast<size_t>(b) * hw * c + ch;
    int32_t sum = 0;
    for (int i = 0; i < hw; ++i) sum += p[static_cast<size_t>(i) * c];
    int q = __float2int_rn(__fdiv_rn(static_cast<float>(sum), cnt));
    q = min(max(q, -128), 127);
    y[static_cast<size_t>(b) * c + ch] = static_cast<int8_t>(q);
  }
}

// Packed rows word by word (dilation 1, short rows): row m's packed bytes are R segments of L = S*C contiguous
// input bytes (filter row rr starts at input (hi0 + rr, wi0)), written back to back and followed by
// zeros up to kp.  One thread per row; each output word is two aligned input words and a funnel
// shift when its 4 bytes lie in one segment, bytes otherwise (the few words that straddle two
// segments, and rows whose window leaves the image).  16-byte stores of 4 assembled words.
__global__ void __launch_bounds__(256) im2col_pack_words_kernel(const int8_t* __restrict__ x,
                                                                int8_t* __restrict__ a, ConvGeom g, int kp,
                                                                long long total_rows, size_t x_bytes) {
  // Aligned word pairs are read only where both words lie inside x.
  const uintptr_t x_end = reinterpret_cast<uintptr_t>(x) + x_bytes;
  const int L = g.s * g.c;
  const int rsc = g.r * L;
  for (long long m = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; m < total_rows;
       m += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int wo = static_cast<int>(m % g.wo);
    const long long t = m / g.wo;
    const int ho = static_cast<int>(t % g.ho);
    const int n = static_cast<int>(t / g.ho);
    const int hi0 = ho * g.stride_h - g.pad_h, wi0 = wo * g.stride_w - g.pad_w;
    const bool inside = hi0 >= 0 && hi0 + g.r <= g.h && wi0 >= 0 && wi0 + g.s <= g.w;
    const int8_t* img = x + static_cast<size_t>(n) * g.h * g.w * g.c;
    uint4* out = reinterpret_cast<uint4*>(a + m * kp);
    int rr = 0, off = 0;  // segment and offset of output byte 4q
    for (int v = 0; v < kp / 16; ++v) {
      uint32_t wd[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = (v * 4 + q) * 4;
        uint32_t word = 0;
        const uintptr_t src =
            reinterpret_cast<uintptr_t>(img + (static_cast<size_t>(hi0 + rr) * g.w + wi0) * g.c + off);
        if (j + 4 <= rsc && off + 4 <= L && inside && (src & ~uintptr_t(3)) + 8 <= x_end) {
          const uint32_t* w0 = reinterpret_cast<const uint32_t*>(src & ~uintptr_t(3));
          const uint32_t sh = static_cast<uint32_t>(src & 3) * 8;
          const uint32_t lo = __ldg(w0);
          const uint32_t hi = sh ? __ldg(w0 + 1) : 0u;
          word = __funnelshift_r(lo, hi, sh);
        } else {
          int r2 = rr, o2 = off;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            if (j + b < rsc) {
              const int ss = o2 / g.c, c = o2 - ss * g.c;
              const int hi = hi0 + r2, wi = wi0 + ss;
              if (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w)
                word |= static_cast<uint32_t>(static_cast<uint8_t>(img[(static_cast<size_t>(hi) * g.w + wi) * g.c + c]))
                        << (8 * b);
            }
            if (++o2 == L) {
              o2 = 0;
              ++r2;
            }
          }
        }
        wd[q] = word;
        off += 4;
        while (off >= L) {
          off -= L;
          ++rr;
        }
      }
      out[v] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
  }
}

// Weights [k][R*S*C] -> [k][kp] with zero columns past R*S*C.
__global__ void weight_pad_s8_kernel(const int8_t* __restrict__ w, int8_t* __restrict__ wp, int k, int rsc, int kp) {
  const size_t total = static_cast<size_t>(k) * kp;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(idx / kp);
    const int col = static_cast<int>(idx - static_cast<size_t>(row) * kp);
    wp[idx] = col < rsc ? w[static_cast<size_t>(row) * rsc + col] : static_cast<int8_t>(0);
  }
}

// Space-to-depth of a stride-2 conv input: x [n][h][w][C] (C <= 4) -> xs [n][h2][w2][16] with
// xs[i][Y][X][(dy * 2 + dx) * C + ci] = x[i][2Y + dy][2X + dx][ci], zero past the image and in
// channels 4C..15.  A stride-2 R x S conv of x is then a stride-1 conv of xs (weights rearranged
// by s2d_weight_s8_kernel) whose 16-byte pixels a TMA box can load.  One thread per output pixel.
template <int C>
__global__ void s2d_s8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ xs, int n, int h, int w, int h2,
                              int w2) {
  const size_t total = static_cast<size_t>(n) * h2 * w2;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int X = static_cast<int>(idx % w2);
    const size_t t = idx / w2;
    const int Y = static_cast<int>(t % h2);
    const int img = static_cast<int>(t / h2);
    uint32_t wd[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int y = 2 * Y + (q >> 1), xx = 2 * X + (q & 1);
      if (y < h && xx < w) {
        const int8_t* src = x + ((static_cast<size_t>(img) * h + y) * w + xx) * C;
#pragma unroll
        for (int ci = 0; ci < C; ++ci) {
          const int byte = q * C + ci;
          wd[byte >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(src[ci])) << (8 * (byte & 3));
        }
      }
    }
    reinterpret_cast<uint4*>(xs)[idx] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

// Weights of a stride-2 conv [k][rk][sk][c] -> [k][r2][s2][16] for the space-to-depth input:
// tap (R, S), channel (dy * 2 + dx) * c + ci holds w[kk][r][s][ci] with
// r = 2 * (R + yoff) + dy + pad_h, s = 2 * (S + xoff) + dx + pad_w (zero outside the filter), where
// yoff = floor(-pad_h / 2), xoff = floor(-pad_w / 2) place the window's first space-to-depth row /
// column relative to the output row / column.
__global__ void s2d_weight_s8_kernel(const int8_t* __restrict__ w, int8_t* __restrict__ ws, int k, int rk, int sk,
                                     int c, int r2, int s2, int pad_h, int pad_w) {
  const int total = k * r2 * s2 * 16;
  const int yoff = -((pad_h + 1) / 2), xoff = -((pad_w + 1) / 2);
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int cc = idx & 15;
    int t = idx >> 4;
    const int S = t % s2;
    t /= s2;
    const int R = t % r2;
    const int kk = t / r2;
    int8_t v = 0;
    if (cc < 4 * c) {
      const int q = cc / c, ci = cc - q * c;
      const int r = 2 * (R + yoff) + (q >> 1) + pad_h, s = 2 * (S + xoff) + (q & 1) + pad_w;
      if (r >= 0 && r < rk && s >= 0 && s < sk) v = w[((static_cast<size_t>(kk) * rk + r) * sk + s) * c + ci];
    }
    ws[idx] = v;
  }
}

}  // namespace b200q
