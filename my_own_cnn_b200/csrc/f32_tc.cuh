// fp32 convolution (fprop / bprop / grad, regular and blocked) and fp32 batched GEMM on the
// tensor cores, for the reference's fp32 entry points (src/cuda_kernels.cu:767-937, 1000-1136;
// bmm.cu:270-361).
//
// Precision: the tensor core's fp32 input format (TF32) keeps 10 mantissa bits, so every operand is
// split as x = hi + lo with hi = x rounded to 10 bits (its low 13 bits zero: the tensor core reads it
// exactly) and lo = x - hi (exact in fp32).  Laying the parts out along the reduction as
//     A' = [hi | hi | lo],   B' = [hi | lo | hi]
// makes one kind::tf32 GEMM over 3K compute sum(hi_a hi_b + hi_a lo_b + lo_a hi_b): only lo_a lo_b
// (below 2^-21 of each product) and lo's own 10-bit read are dropped, so each product is within
// ~2^-20 relative of fp32 and the accumulation is fp32 in TMEM.
//
// Every operation is one batched GEMM between two packed operands.  f32_pack_kernel builds them
// from the caller's tensors: it reads a 32 x 32 tile of the logical matrix (rows x reduction) in
// whichever direction is contiguous in memory, transposes through shared memory, and writes the
// three split thirds row by row.  The logical matrices (batch item b = (split, block, group)):
//   fprop  A[p][j] = im2col(x)          B[k][j] = w[k][block][j]          C[p][k]  -> y
//   bprop  A[p][k] = dy                 B[j][k] = w[k][block][j]          C[p][j]  -> col2im -> dx
//   grad   A[k][p] = dy (transposed)    B[j][p] = im2col(x) (transposed)  C[k][j]  -> sum of splits -> dw
//   bmm    A = op(A), B = op(B)^T from the strided source                 C        -> C
// with p an output pixel of the block, j = (r, s, c) a tap x input channel of the group, k an
// output channel of the group.  The post-passes are gathers (each output element written once,
// deterministic).
#pragma once
#include "simt.cuh"

namespace b200q {

// x = hi + lo, hi with the low 13 mantissa bits zero (round to nearest on the 10-bit mantissa).
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
  hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
  lo = __fsub_rn(x, hi);
}

enum F32PackMode {
  kPackMat = 0,         // element (b, r, c) at src[b * sb + r * sr + c * sc]
  kPackIm2colRows = 1,  // fprop A: r = pixel, c = tap x channel
  kPackIm2colCols = 2,  // grad B:  r = tap x channel, c = pixel
  kPackDyRows = 3,      // bprop A: r = pixel, c = output channel of the group
  kPackDyCols = 4,      // grad A:  r = output channel, c = pixel
  kPackWRows = 5,       // fprop B: r = output channel, c = tap x channel
  kPackWCols = 6,       // bprop B: r = tap x channel, c = output channel
};

struct F32Pack {
  int mode;
  int rows, cols;  // logical matrix per batch item
  int kp;          // packed third: cols rounded up to 32
  int lo_mask;     // bit i: third i holds lo parts (A: 4 = [hi|hi|lo], B: 2 = [hi|lo|hi])
  int batch;
  long long sb, sr, sc;  // kPackMat strides (elements)
  ConvGeom g;
  int T;           // taps x channels of a group: R * S * Cg
  int nblk;        // output blocks: By * Bx
  int mb;          // pixels per block item: N * bho * bwo
  int chunk;       // pixels per reduction split (grad); mb for the other modes
};

// Output pixel p of block blk -> (n, ho, wo).
__device__ __forceinline__ void f32_pixel(const ConvGeom& g, int blk, int p, int& n, int& ho, int& wo) {
  const int owb = p % g.bwo;
  const int t = p / g.bwo;
  const int ohb = t % g.bho;
  n = t / g.bho;
  const int byi = blk / g.bx, bxi = blk - byi * g.bx;
  ho = byi * g.bho + ohb;
  wo = bxi * g.bwo + owb;
}

// x value of tap x channel j at output pixel (n, ho, wo) of group grp (0 in the padding).
__device__ __forceinline__ float f32_im2col(const float* x, const ConvGeom& g, int grp, int n, int ho, int wo, int j) {
  const int c = j % g.cg;
  const int t = j / g.cg;
  const int s = t % g.s, r = t / g.s;
  const int hi = ho * g.stride_h - g.pad_h + r * g.dil_h;
  const int wi = wo * g.stride_w - g.pad_w + s * g.dil_w;
  if (hi < 0 || hi >= g.h || wi < 0 || wi >= g.w) return 0.0f;
  return __ldg(x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + static_cast<size_t>(grp) * g.cg + c);
}

// Logical element (b, r, c); c < cols and r < rows are guaranteed by the caller.
__device__ __forceinline__ float f32_value(const float* src, const F32Pack& q, int b, int r, int c) {
  if (q.mode == kPackMat) return __ldg(src + b * q.sb + r * q.sr + c * q.sc);
  const ConvGeom& g = q.g;
  const int G = g.groups;
  const int grp = b % G;
  const int blk = (b / G) % q.nblk;
  const int split = b / (G * q.nblk);
  switch (q.mode) {
    case kPackIm2colRows: {
      int n, ho, wo;
      f32_pixel(g, blk, r, n, ho, wo);
      return f32_im2col(src, g, grp, n, ho, wo, c);
    }
    case kPackIm2colCols: {
      const int p = split * q.chunk + c;
      if (p >= q.mb) return 0.0f;
      int n, ho, wo;
      f32_pixel(g, blk, p, n, ho, wo);
      return f32_im2col(src, g, grp, n, ho, wo, r);
    }
    case kPackDyRows: {
      int n, ho, wo;
      f32_pixel(g, blk, r, n, ho, wo);
      return __ldg(src + ((static_cast<size_t>(n) * g.ho + ho) * g.wo + wo) * g.k + grp * g.kg + c);
    }
    case kPackDyCols: {
      const int p = split * q.chunk + c;
      if (p >= q.mb) return 0.0f;
      int n, ho, wo;
      f32_pixel(g, blk, p, n, ho, wo);
      return __ldg(src + ((static_cast<size_t>(n) * g.ho + ho) * g.wo + wo) * g.k + grp * g.kg + r);
    }
    case kPackWRows:  // w[k][block][j], k = grp * Kg + r
      return __ldg(src + (static_cast<size_t>(grp * g.kg + r) * q.nblk + blk) * q.T + c);
    default:  // kPackWCols: w[k][block][j], k = grp * Kg + c, j = r
      return __ldg(src + (static_cast<size_t>(grp * g.kg + c) * q.nblk + blk) * q.T + r);
  }
}

// Whether consecutive rows (rather than columns) of the logical matrix are contiguous in memory.
__host__ __device__ inline bool f32_rows_contiguous(const F32Pack& q) {
  return q.mode == kPackIm2colCols || q.mode == kPackDyCols || q.mode == kPackWCols ||
         (q.mode == kPackMat && q.sr == 1 && q.sc != 1);
}

// Split-pack of a 32 x 32 tile: dst[b][r][third * kp + c], zero for c >= cols.  256 threads.
__global__ void __launch_bounds__(256) f32_pack_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                       F32Pack q) {
  __shared__ float tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int ctiles = q.kp / 32;
  const int rtiles = (q.rows + 31) / 32;
  const long long total = static_cast<long long>(q.batch) * rtiles * ctiles;
  const bool rows_contig = f32_rows_contiguous(q);
  for (long long t = blockIdx.x; t < total; t += gridDim.x) {
    const int ct = static_cast<int>(t % ctiles);
    const long long t2 = t / ctiles;
    const int rt = static_cast<int>(t2 % rtiles);
    const int b = static_cast<int>(t2 / rtiles);
    const int r0 = rt * 32, c0 = ct * 32;
    // load: lanes run along the contiguous direction
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int a = ty + 8 * i;  // the other direction
      const int r = rows_contig ? r0 + tx : r0 + a;
      const int c = rows_contig ? c0 + a : c0 + tx;
      float v = 0.0f;
      if (r < q.rows && c < q.cols) v = f32_value(src, q, b, r, c);
      if (rows_contig)
        tile[tx][a] = v;
      else
        tile[a][tx] = v;
    }
    __syncthreads();
    // store: lanes along the packed row (columns), three thirds
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = ty + 8 * i;
      const int r = r0 + rr;
      if (r < q.rows) {
        float hi, lo;
        tf32_split(tile[rr][tx], hi, lo);
        float* d = dst + (static_cast<size_t>(b) * q.rows + r) * (3 * static_cast<size_t>(q.kp)) + c0 + tx;
        d[0] = (q.lo_mask & 1) ? lo : hi;
        d[q.kp] = (q.lo_mask & 2) ? lo : hi;
        d[2 * q.kp] = (q.lo_mask & 4) ? lo : hi;
      }
    }
    __syncthreads();
  }
}

// fprop post-pass: y[n][ho][wo][k] = C[b][p][kg] (+ bias of the output block).  bias_mode 0 = one
// bias per (k, block), 1 = one per k shared by all blocks (BlockBiasMode, src/conv_types.h:36-39).
__global__ void f32_fprop_scatter_kernel(const float* __restrict__ cbuf, float* __restrict__ y, ConvGeom g, int mb,
                                         const float* __restrict__ bias, int bias_mode) {
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int kk = static_cast<int>(idx % g.k);
    size_t pix = idx / g.k;
    const int wo = static_cast<int>(pix % g.wo);
    pix /= g.wo;
    const int ho = static_cast<int>(pix % g.ho);
    const int n = static_cast<int>(pix / g.ho);
    const int grp = kk / g.kg, kg = kk - grp * g.kg;
    const int byi = ho / g.bho, bxi = wo / g.bwo;
    const int blk = byi * g.bx + bxi;
    const int p = (n * g.bho + (ho - byi * g.bho)) * g.bwo + (wo - bxi * g.bwo);
    float v = __ldg(cbuf + ((static_cast<size_t>(blk) * g.groups + grp) * mb + p) * g.kg + kg);
    // bias index of BlockBiasMode (src/conv_types.h:184-188): (k * By + by) * Bx + bx per block, k * By * Bx shared
    if (bias)
      v = __fadd_rn(v, __ldg(bias + static_cast<size_t>(kk) * g.by * g.bx + (bias_mode == 0 ? blk : 0)));
    y[idx] = v;
  }
}

// bprop post-pass (col2im as a gather): dx[n][hi][wi][grp * Cg + c] = sum over the taps (r, s) whose
// output pixel (ho, wo) exists of col[b(ho, wo)][p(ho, wo)][(r * S + s) * Cg + c]; the same validity
// rule as the reference (src/cpu_ref.cpp:150-192).
__global__ void f32_col2im_kernel(const float* __restrict__ col, float* __restrict__ dx, ConvGeom g, int mb, int T) {
  const size_t total = static_cast<size_t>(g.n) * g.h * g.w * g.c;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int cc = static_cast<int>(idx % g.c);
    size_t pix = idx / g.c;
    const int wi = static_cast<int>(pix % g.w);
    pix /= g.w;
    const int hi = static_cast<int>(pix % g.h);
    const int n = static_cast<int>(pix / g.h);
    const int grp = cc / g.cg, c = cc - grp * g.cg;
    float acc = 0.0f;
    for (int r = 0; r < g.r; ++r) {
      const int hn = hi + g.pad_h - r * g.dil_h;
      if (hn < 0 || hn % g.stride_h) continue;
      const int ho = hn / g.stride_h;
      if (ho >= g.ho) continue;
      for (int s = 0; s < g.s; ++s) {
        const int wn = wi + g.pad_w - s * g.dil_w;
        if (wn < 0 || wn % g.stride_w) continue;
        const int wo = wn / g.stride_w;
        if (wo >= g.wo) continue;
        const int byi = ho / g.bho, bxi = wo / g.bwo;
        const int blk = byi * g.bx + bxi;
        const int p = (n * g.bho + (ho - byi * g.bho)) * g.bwo + (wo - bxi * g.bwo);
        acc = __fadd_rn(acc, __ldg(col + ((static_cast<size_t>(blk) * g.groups + grp) * mb + p) * T +
                                   (r * g.s + s) * g.cg + c));
      }
    }
    dx[idx] = acc;
  }
}

// grad post-pass: dw[k][block][j] = sum over reduction splits of C[split][block][grp][kg][j].
__global__ void f32_grad_reduce_kernel(const float* __restrict__ cbuf, float* __restrict__ dw, ConvGeom g, int nblk,
                                       int T, int splits) {
  const size_t total = static_cast<size_t>(g.k) * nblk * T;
  const size_t split_stride = static_cast<size_t>(nblk) * g.groups * g.kg * T;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % T);
    const size_t t = idx / T;
    const int blk = static_cast<int>(t % nblk);
    const int kk = static_cast<int>(t / nblk);
    const int grp = kk / g.kg, kg = kk - grp * g.kg;
    const float* cp = cbuf + ((static_cast<size_t>(blk) * g.groups + grp) * g.kg + kg) * T + j;
    float acc = 0.0f;
    for (int sp = 0; sp < splits; ++sp) acc = __fadd_rn(acc, __ldg(cp + sp * split_stride));
    dw[idx] = acc;
  }
}

// Blocked grad's bias gradient, the reference's rule (src/cpu_ref.cpp:318-371): dy summed over the
// block's output pixels whose tap (0, 0) input lies inside the image.  The array has K * By * Bx
// entries in both modes; bias_mode 1 (shared) sums all blocks into entry k * By * Bx and leaves the
// others zero.  One CTA per entry, fixed-order tree reduction.
__global__ void __launch_bounds__(256) f32_dbias_kernel(const float* __restrict__ dy, float* __restrict__ dbias,
                                                        ConvGeom g, int bias_mode) {
  __shared__ float red[256];
  const int nblk = g.by * g.bx;
  const int entries = g.k * nblk;
  for (int e = blockIdx.x; e < entries; e += gridDim.x) {
    const int kk = e / nblk, eb = e % nblk;
    int b0 = eb, b1 = eb + 1;
    if (bias_mode != 0) {
      b0 = 0;
      b1 = eb == 0 ? nblk : 0;  // only entry k * By * Bx receives the sum
    }
    const int per = g.n * g.bho * g.bwo;
    float acc = 0.0f;
    for (int blk = b0; blk < b1; ++blk)
      for (int p = threadIdx.x; p < per; p += blockDim.x) {
        int n, ho, wo;
        f32_pixel(g, blk, p, n, ho, wo);
        const int hi = ho * g.stride_h - g.pad_h, wi = wo * g.stride_w - g.pad_w;
        if (hi < 0 || hi >= g.h || wi < 0 || wi >= g.w) continue;
        acc = __fadd_rn(acc, __ldg(dy + ((static_cast<size_t>(n) * g.ho + ho) * g.wo + wo) * g.k + kk));
      }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + o]);
      __syncthreads();
    }
    if (threadIdx.x == 0) dbias[e] = red[0];
    __syncthreads();
  }
}

// ---- fp32 convs through the im2col TMA (groups == 1, no blocks): the input is split once into hi
// and lo copies (which stay in L2 for typical sizes) and the tensor core reads the taps straight
// from them, three passes over the taps ([hi | hi | lo] against packed weights [hi | lo | hi]).

__global__ void f32_split_kernel(const float4* __restrict__ x, float4* __restrict__ hi, float4* __restrict__ lo,
                                 size_t n4) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 v = __ldg(x + i);
    float4 h, l;
    tf32_split(v.x, h.x, l.x);
    tf32_split(v.y, h.y, l.y);
    tf32_split(v.z, h.z, l.z);
    tf32_split(v.w, h.w, l.w);
    hi[i] = h;
    lo[i] = l;
  }
}

// Packed weights for the im2col-TMA conv: row k' of 3 x L floats, L = R * S * cpad (the group's
// cin channels padded to cpad, a multiple of 32 = one 128-byte K block), thirds [hi | lo | hi].
// flip = 0: the conv's own filter [kout][R][S][cin] (row k', channel c).  flip = 1: the data-gradient
// filter of a stride-1 conv: row k' is input channel k' of the forward conv, in group
// grp = k' / kout_g; its channel c is the forward conv's output channel grp * cin + c, and
// w'[k'][r][s][c] = w[grp * cin + c][R-1-r][S-1-s][k' - grp * kout_g] (forward filter [K][R][S][kout_g]).
__global__ void f32_pack_taps_kernel(const float* __restrict__ w, float* __restrict__ dst, int kout, int r, int s,
                                     int cin, int cpad, int flip, int kout_g) {
  const int L = r * s * cpad;
  const size_t total = static_cast<size_t>(kout) * 3 * L;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % (3 * L));
    const int kp = static_cast<int>(idx / (3 * L));
    const int third = j / L, jj = j - third * L;
    const int tap = jj / cpad, c = jj - tap * cpad;
    float v = 0.0f;
    if (c < cin) {
      const int rr = tap / s, ss = tap - rr * s;
      if (flip) {
        const int grp = kp / kout_g;
        v = __ldg(w + ((static_cast<size_t>(grp * cin + c) * r + (r - 1 - rr)) * s + (s - 1 - ss)) * kout_g +
                  (kp - grp * kout_g));
      } else {
        v = __ldg(w + ((static_cast<size_t>(kp) * r + rr) * s + ss) * cin + c);
      }
    }
    float hi, lo;
    tf32_split(v, hi, lo);
    dst[idx] = third == 1 ? lo : hi;
  }
}

// ---- direct CUDA-core kernels for groups of a few channels (depthwise and the like), where a GEMM
// per group would have 1-4 rows or columns.  The loops are the reference's (src/cpu_ref.cpp:116-371)
// with fp32 fused multiply-adds.

// y element per thread (+ block bias).
__global__ void f32_direct_fprop_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                        float* __restrict__ y, ConvGeom g, const float* __restrict__ bias,
                                        int bias_mode) {
  const size_t total = static_cast<size_t>(g.n) * g.ho * g.wo * g.k;
  const int nblk = g.by * g.bx, T = g.r * g.s * g.cg;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int kk = static_cast<int>(idx % g.k);
    size_t pix = idx / g.k;
    const int wo = static_cast<int>(pix % g.wo);
    pix /= g.wo;
    const int ho = static_cast<int>(pix % g.ho);
    const int n = static_cast<int>(pix / g.ho);
    const int grp = kk / g.kg;
    const int blk = (ho / g.bho) * g.bx + wo / g.bwo;
    const float* wp = w + (static_cast<size_t>(kk) * nblk + blk) * T;
    float acc = 0.0f;
    for (int r = 0; r < g.r; ++r) {
      const int hi = ho * g.stride_h - g.pad_h + r * g.dil_h;
      if (hi < 0 || hi >= g.h) continue;
      for (int s = 0; s < g.s; ++s) {
        const int wi = wo * g.stride_w - g.pad_w + s * g.dil_w;
        if (wi < 0 || wi >= g.w) continue;
        const float* xp = x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + grp * g.cg;
        const float* wq = wp + (r * g.s + s) * g.cg;
        for (int c = 0; c < g.cg; ++c) acc = __fmaf_rn(__ldg(xp + c), __ldg(wq + c), acc);
      }
    }
    if (bias) acc = __fadd_rn(acc, __ldg(bias + static_cast<size_t>(kk) * nblk + (bias_mode == 0 ? blk : 0)));
    y[idx] = acc;
  }
}

// dx element per thread.
__global__ void f32_direct_bprop_kernel(const float* __restrict__ dy, const float* __restrict__ w,
                                        float* __restrict__ dx, ConvGeom g) {
  const size_t total = static_cast<size_t>(g.n) * g.h * g.w * g.c;
  const int nblk = g.by * g.bx, T = g.r * g.s * g.cg;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int cc = static_cast<int>(idx % g.c);
    size_t pix = idx / g.c;
    const int wi = static_cast<int>(pix % g.w);
    pix /= g.w;
    const int hi = static_cast<int>(pix % g.h);
    const int n = static_cast<int>(pix / g.h);
    const int grp = cc / g.cg, c = cc - grp * g.cg;
    float acc = 0.0f;
    for (int r = 0; r < g.r; ++r) {
      const int hn = hi + g.pad_h - r * g.dil_h;
      if (hn < 0 || hn % g.stride_h) continue;
      const int ho = hn / g.stride_h;
      if (ho >= g.ho) continue;
      for (int s = 0; s < g.s; ++s) {
        const int wn = wi + g.pad_w - s * g.dil_w;
        if (wn < 0 || wn % g.stride_w) continue;
        const int wo = wn / g.stride_w;
        if (wo >= g.wo) continue;
        const int blk = (ho / g.bho) * g.bx + wo / g.bwo;
        const float* dyp = dy + ((static_cast<size_t>(n) * g.ho + ho) * g.wo + wo) * g.k + grp * g.kg;
        for (int kg = 0; kg < g.kg; ++kg)
          acc = __fmaf_rn(__ldg(dyp + kg),
                          __ldg(w + (static_cast<size_t>(grp * g.kg + kg) * nblk + blk) * T + (r * g.s + s) * g.cg + c),
                          acc);
      }
    }
    dx[idx] = acc;
  }
}

// dw element per CTA: the block's output pixels are split over the threads, then a fixed-order
// tree reduction.
__global__ void __launch_bounds__(256) f32_direct_grad_kernel(const float* __restrict__ x, const float* __restrict__ dy,
                                                              float* __restrict__ dw, ConvGeom g) {
  __shared__ float red[256];
  const int nblk = g.by * g.bx, T = g.r * g.s * g.cg;
  const long long total = static_cast<long long>(g.k) * nblk * T;
  const int per = g.n * g.bho * g.bwo;
  for (long long e = blockIdx.x; e < total; e += gridDim.x) {
    const int j = static_cast<int>(e % T);
    const long long t = e / T;
    const int blk = static_cast<int>(t % nblk);
    const int kk = static_cast<int>(t / nblk);
    const int grp = kk / g.kg;
    const int c = j % g.cg, tap = j / g.cg;
    const int s = tap % g.s, r = tap / g.s;
    float acc = 0.0f;
    for (int p = threadIdx.x; p < per; p += blockDim.x) {
      int n, ho, wo;
      f32_pixel(g, blk, p, n, ho, wo);
      const int hi = ho * g.stride_h - g.pad_h + r * g.dil_h;
      const int wi = wo * g.stride_w - g.pad_w + s * g.dil_w;
      if (hi < 0 || hi >= g.h || wi < 0 || wi >= g.w) continue;
      acc = __fmaf_rn(__ldg(x + ((static_cast<size_t>(n) * g.h + hi) * g.w + wi) * g.c + grp * g.cg + c),
                      __ldg(dy + ((static_cast<size_t>(n) * g.ho + ho) * g.wo + wo) * g.k + kk), acc);
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] = __fadd_rn(red[threadIdx.x], red[threadIdx.x + o]);
      __syncthreads();
    }
    if (threadIdx.x == 0) dw[e] = red[0];
    __syncthreads();
  }
}

}  // namespace b200q
