// C entry points over the reference's own CPU oracle (test infrastructure only).
//
// Compiled together with the reference's unmodified src/cpu_ref.cpp (and its
// headers src/conv_types.h, src/nnalgebra_quantization.h) by oracle/Makefile
// into oracle/_ref/libref_oracle.so.  Nothing from the reference is copied:
// this file only builds the reference's tensor structs from flat buffers and
// calls cpu_fprop_nhwc_qi32 / cpu_block_fprop_nhwc_qi32
// (conv_types.h:255-285, cpu_ref.cpp:36-112, exports cpu_ref.cpp:371-401) and the fp32
// cpu_{,block_}{fprop,bprop,grad}_nhwc (conv_types.h:204-210, cpu_ref.cpp:116-371).
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

#include "conv_types.h"

namespace {

using U8 = nnalgebra::QuantizationParameters<nnalgebra::DataType::LinQuantU8>;
using S5 = nnalgebra::QuantizationParameters<nnalgebra::DataType::LinQuantS5>;

struct Args {
  int n, h, w, c, r, s, k;
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w, groups;
  int by, bx;
};

Conv2DParams to_params(const Args& a) {
  Conv2DParams p;
  p.pad_h = a.pad_h;
  p.pad_w = a.pad_w;
  p.stride_h = a.stride_h;
  p.stride_w = a.stride_w;
  p.dilation_h = a.dil_h;
  p.dilation_w = a.dil_w;
  p.groups = a.groups;
  return p;
}

// kind 0 = LinQuantU8, 1 = LinQuantS5.  zp_in: per image, zp_f: filter.
int run(const Args& a, int kind, int blocked, const float* x, const float* w, int32_t* y,
        const int32_t* zp_in, int32_t zp_f) {
  try {
    TensorNHWC xt(a.n, a.h, a.w, a.c);
    std::memcpy(xt.ptr(), x, xt.elements() * sizeof(float));
    TensorNHWCI32 yt;
    const Conv2DParams p = to_params(a);
    if (!blocked) {
      FilterKRSC wt(a.r, a.s, a.c / a.groups, a.k);
      std::memcpy(wt.ptr(), w, wt.elements() * sizeof(float));
      if (kind == 0) {
        std::vector<U8> iq(a.n);
        for (int i = 0; i < a.n; ++i) iq[i].zero_point = static_cast<uint8_t>(zp_in[i]);
        U8 fq;
        fq.zero_point = static_cast<uint8_t>(zp_f);
        cpu_fprop_nhwc_qi32<nnalgebra::DataType::LinQuantU8>(xt, wt, p, yt, iq.data(), &fq);
      } else {
        std::vector<S5> iq(a.n);
        for (int i = 0; i < a.n; ++i) iq[i].zero_point = static_cast<int8_t>(zp_in[i]);
        S5 fq;
        fq.zero_point = static_cast<int8_t>(zp_f);
        cpu_fprop_nhwc_qi32<nnalgebra::DataType::LinQuantS5>(xt, wt, p, yt, iq.data(), &fq);
      }
    } else {
      BlockConv2DParams bp;
      bp.conv = p;
      bp.block_by = a.by;
      bp.block_bx = a.bx;
      BlockFilterKByBxRSC wt(a.k, a.by, a.bx, a.r, a.s, a.c / a.groups);
      std::memcpy(wt.ptr(), w, wt.elements() * sizeof(float));
      if (kind == 0) {
        std::vector<U8> iq(a.n);
        for (int i = 0; i < a.n; ++i) iq[i].zero_point = static_cast<uint8_t>(zp_in[i]);
        U8 fq;
        fq.zero_point = static_cast<uint8_t>(zp_f);
        cpu_block_fprop_nhwc_qi32<nnalgebra::DataType::LinQuantU8>(xt, wt, bp, yt, iq.data(), &fq);
      } else {
        std::vector<S5> iq(a.n);
        for (int i = 0; i < a.n; ++i) iq[i].zero_point = static_cast<int8_t>(zp_in[i]);
        S5 fq;
        fq.zero_point = static_cast<int8_t>(zp_f);
        cpu_block_fprop_nhwc_qi32<nnalgebra::DataType::LinQuantS5>(xt, wt, bp, yt, iq.data(), &fq);
      }
    }
    std::memcpy(y, yt.ptr(), yt.elements() * sizeof(int32_t));
    return 0;
  } catch (const std::exception&) {
    return 1;  // the reference threw std::runtime_error (shape validation)
  }
}

}  // namespace

extern "C" {

int ref_fprop_qi32(const Args* a, int kind, int blocked, const float* x, const float* w, int32_t* y,
                   const int32_t* zp_in, int32_t zp_f) {
  return run(*a, kind, blocked, x, w, y, zp_in, zp_f);
}

// Batch split over threads, each calling the reference oracle on its slice of
// images (exact: images are independent).  Used as the timed CPU baseline.
int ref_fprop_qi32_threaded(const Args* a, int kind, const float* x, const float* w, int32_t* y,
                            const int32_t* zp_in, int32_t zp_f, int threads) {
  int ho = 0, wo = 0;
  {
    const int hn = a->h + 2 * a->pad_h - a->dil_h * (a->r - 1) - 1;
    const int wn = a->w + 2 * a->pad_w - a->dil_w * (a->s - 1) - 1;
    if (hn < 0 || wn < 0 || a->stride_h <= 0 || a->stride_w <= 0) return 1;
    ho = hn / a->stride_h + 1;
    wo = wn / a->stride_w + 1;
  }
  if (threads < 1) threads = 1;
  if (threads > a->n) threads = a->n;
  const size_t x_img = static_cast<size_t>(a->h) * a->w * a->c;
  const size_t y_img = static_cast<size_t>(ho) * wo * a->k;
  std::vector<std::thread> pool;
  std::vector<int> rc(threads, 0);
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t]() {
      const int n0 = static_cast<int>(static_cast<long long>(a->n) * t / threads);
      const int n1 = static_cast<int>(static_cast<long long>(a->n) * (t + 1) / threads);
      if (n1 <= n0) return;
      Args s = *a;
      s.n = n1 - n0;
      rc[t] = run(s, kind, 0, x + x_img * n0, w, y + y_img * n0, zp_in + n0, zp_f);
    });
  }
  for (auto& th : pool) th.join();
  for (int v : rc)
    if (v) return v;
  return 0;
}

// The reference's fp32 CPU loops.  op 0 = fprop (a = x, b = w, out = y), 1 = bprop (a = dy,
// b = w, out = dx), 2 = grad (a = x, b = dy, out = dw).  Blocked when a->by * a->bx > 1 or
// blocked != 0; bias / dbias (K * By * Bx floats, may be null) with bias_mode as BlockBiasMode.
int ref_conv_f32(const Args* a, int op, int blocked, const float* in_a, const float* in_b, float* out,
                 float* bias, int bias_mode) {
  try {
    const Conv2DParams p = to_params(*a);
    const int cg = a->c / a->groups;
    TensorNHWC x(a->n, a->h, a->w, a->c);
    FilterKRSC wshape(a->r, a->s, cg, a->k);
    const ConvShape sh = infer_conv_shape(x, wshape, p);
    TensorNHWC y(a->n, sh.ho, sh.wo, a->k);
    BlockConv2DParams bp;
    bp.conv = p;
    bp.block_by = a->by;
    bp.block_bx = a->bx;
    const BlockBiasMode mode = bias_mode ? BlockBiasMode::Shared : BlockBiasMode::PerBlock;
    if (!blocked) {
      FilterKRSC w(a->r, a->s, cg, a->k);
      if (op == 0) {
        std::memcpy(x.ptr(), in_a, x.elements() * sizeof(float));
        std::memcpy(w.ptr(), in_b, w.elements() * sizeof(float));
        cpu_fprop_nhwc(x, w, p, y);
        std::memcpy(out, y.ptr(), y.elements() * sizeof(float));
      } else if (op == 1) {
        std::memcpy(y.ptr(), in_a, y.elements() * sizeof(float));
        std::memcpy(w.ptr(), in_b, w.elements() * sizeof(float));
        cpu_bprop_nhwc(y, w, p, x);
        std::memcpy(out, x.ptr(), x.elements() * sizeof(float));
      } else {
        std::memcpy(x.ptr(), in_a, x.elements() * sizeof(float));
        std::memcpy(y.ptr(), in_b, y.elements() * sizeof(float));
        cpu_grad_nhwc(x, y, p, w);
        std::memcpy(out, w.ptr(), w.elements() * sizeof(float));
      }
    } else {
      BlockFilterKByBxRSC w(a->k, a->by, a->bx, a->r, a->s, cg);
      if (op == 0) {
        std::memcpy(x.ptr(), in_a, x.elements() * sizeof(float));
        std::memcpy(w.ptr(), in_b, w.elements() * sizeof(float));
        cpu_block_fprop_nhwc(x, w, bp, y, bias, mode);
        std::memcpy(out, y.ptr(), y.elements() * sizeof(float));
      } else if (op == 1) {
        std::memcpy(y.ptr(), in_a, y.elements() * sizeof(float));
        std::memcpy(w.ptr(), in_b, w.elements() * sizeof(float));
        cpu_block_bprop_nhwc(y, w, bp, x);
        std::memcpy(out, x.ptr(), x.elements() * sizeof(float));
      } else {
        std::memcpy(x.ptr(), in_a, x.elements() * sizeof(float));
        std::memcpy(y.ptr(), in_b, y.elements() * sizeof(float));
        cpu_block_grad_nhwc(x, y, bp, w, bias, mode);
        std::memcpy(out, w.ptr(), w.elements() * sizeof(float));
      }
    }
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}

}  // extern "C"
