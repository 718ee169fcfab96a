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

// Depthwise int8 conv (groups == C == K): one thread = one output pixel x 16 channels.
// Weights [C][R][S] are staged transposed as [R*S][C] in shared memory.
__global__ void dw_conv_s8_kernel(const int8_t* __restrict__ x, const int8_t* __restrict__ w,
                                  void* __restrict__ y, ConvGeom g, Epilogue e) {
  extern __shared__ __align__(16) int8_t wsm[];  // [r*s][c]
  const int taps = g.r * g.s;
  for (int i = threadIdx.x; i < taps * g.c; i += blockDim.x) {
    const int ch = i % g.c, t = i / g.c;
    wsm[i] = w[static_cast<size_t>(ch) * taps + t];
  }
  __syncthreads();
  const int cgroups = g.c >> 4;
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * cgroups;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int cgi = static_cast<int>(idx % cgroups);
    size_t pix = idx / cgroups;
    const int wo = static_cast<int>(pix % g.wo);
    pix /= g.wo;
    const int ho = static_cast<int>(pix % g.ho);
    const int n = static_cast<int>(pix / g.ho);
    const int c0 = cgi << 4;
    int32_t acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0;
    for (int rr = 0; rr < g.r; ++rr) {
      const int hi = ho * g.stride_h - g.pad_h + rr * g.dil_h;
      if (hi < 0 || hi >= g.h) continue;
      for (int ss = 0; ss < g.s; ++ss) {
        const int wi = wo * g.stride_w - g.pad_w + ss * g.dil_w;
        if (wi < 0 || wi >= g.w) continue;
        const int4 xv = __ldg(reinterpret_cast<const int4*>(x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + c0));
        const int4 wv = *reinterpret_cast<const int4*>(wsm + (rr * g.s + ss) * g.c + c0);
        const int xa[4] = {xv.x, xv.y, xv.z, xv.w};
        const int wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int xb = static_cast<int>(static_cast<uint32_t>(xa[q]) << (24 - 8 * b)) >> 24;  // sign-extended byte b
            const int wb = static_cast<int>(static_cast<uint32_t>(wa[q]) << (24 - 8 * b)) >> 24;
            acc[4 * q + b] += xb * wb;
          }
      }
    }
    const size_t obase = idx << 4;  // == ((n*ho + ho)*wo + wo)*C + c0
    if (e.out_kind == kOutS8) {
      uint32_t pk[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int ch = c0 + 4 * q + b;
          const int32_t t = e.bias ? wrap_add(acc[4 * q + b], __ldg(e.bias + ch)) : acc[4 * q + b];
          word |= (static_cast<uint32_t>(requant_one(t, __ldg(e.scale + ch), e)) & 0xFFu) << (8 * b);
        }
        pk[q] = word;
      }
      *reinterpret_cast<int4*>(static_cast<int8_t*>(y) + obase) = make_int4(pk[0], pk[1], pk[2], pk[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) epilogue_store(e, y, obase + j, acc[j], c0 + j);
    }
  }
}

// Tiled batched GEMM on CUDA cores: 64x64 output tile per 256 threads, 4x4 per thread, BK=16.
// C_b = op(A_b) @ op(B_b) with bmm.h:9-29 layouts; products and sums in uint32 (wrap-around),
// which is bmm.cu:218-229's int32 arithmetic without signed-overflow UB.
template <typename T>
__global__ void __launch_bounds__(256) bmm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                       void* __restrict__ C, int M, int N, int K,
                                                       int ta, int tb, Epilogue e) {
  __shared__ int32_t As[16][64 + 1];
  __shared__ int32_t Bs[16][64 + 1];
  const int b = blockIdx.z;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
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
// One thread writes 4 consecutive bytes of a row.
__global__ void im2col_pack_s8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ a, ConvGeom g, int kp,
                                      long long rows) {
  const int words = kp >> 2;
  const int rsc = g.r * g.s * g.c;
  const size_t total = static_cast<size_t>(rows) * words;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const long long m = static_cast<long long>(idx / words);
    const int k0 = static_cast<int>(idx - static_cast<size_t>(m) * words) * 4;
    const int wo = static_cast<int>(m % g.wo);
    const long long t = m / g.wo;
    const int ho = static_cast<int>(t % g.ho);
    const int n = static_cast<int>(t / g.ho);
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int kk = k0 + b;
      if (kk < rsc) {
        const int c = kk % g.c;
        const int tap = kk / g.c;
        const int ss = tap % g.s, rr = tap / g.s;
        const int hi = ho * g.stride_h - g.pad_h + rr * g.dil_h;
        const int wi = wo * g.stride_w - g.pad_w + ss * g.dil_w;
        if (hi >= 0 && hi < g.h && wi >= 0 && wi < g.w) {
          const int8_t v = __ldg(x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + c);
          word |= (static_cast<uint32_t>(static_cast<uint8_t>(v))) << (8 * b);
        }
      }
    }
    reinterpret_cast<uint32_t*>(a)[idx] = word;
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

}  // namespace b200q
