// Shared definitions of the b200q CUDA library: epilogue semantics, device error codes.
#pragma once
#include <cstdint>

namespace b200q {

constexpr int kOutS32 = 0;
constexpr int kOutS8 = 1;
constexpr int kOutF32 = 2;

// Device error word values (first writer wins).
constexpr int kDevErrTimeoutProducer = 0x101;
constexpr int kDevErrTimeoutMma = 0x102;
constexpr int kDevErrTimeoutEpilogue = 0x103;
constexpr int kDevErrTimeoutProbe = 0x104;
constexpr int kDevErrTimeoutDw = 0x105;

struct Epilogue {
  int out_kind;
  int zp;
  int lo;  // clamp bounds in the output code domain
  int hi;
  const int32_t* bias;  // may be null
  const float* scale;   // required for S8 / F32
  const int8_t* res;    // int8 residual with the output's layout (S8 outputs only), or null
  float res_scale;
  // int32 outputs only: per-row terms, t = acc + rowterm[m] - rowzx[m] * bias[col] instead of
  // acc + bias[col] (the quantized-int32 drop-in's zero-point correction; null otherwise)
  const int32_t* rowterm;
  const int32_t* rowzx;
};

// Requantize one int32 value (bias already added, wrapping):
//   p = (float)t * scale          (both IEEE round-to-nearest-even, no contraction)
//   r = rint_sat(p)               (cvt.rni.s32.f32: half to even, saturating, NaN -> 0)
//   q = clamp(r, lo - zp, hi - zp) + zp
// The bounds are integers, so clamping after rounding equals rounding after clamping.
__device__ __forceinline__ int requant_one(int32_t t, float sc, const Epilogue& e) {
  const int r = __float2int_rn(__fmul_rn(__int2float_rn(t), sc));
  return min(max(r, e.lo - e.zp), e.hi - e.zp) + e.zp;
}

// Requantize with a fused residual add (int8 residual code rv, its scale rs):
//   p = fl(fl(t) * scale) + fl(rv * rs)   (three IEEE round-to-nearest-even operations, no fma)
//   q = clamp(rint_sat(p), lo - zp, hi - zp) + zp
__device__ __forceinline__ int requant_res(int32_t t, float sc, int rv, float rs, const Epilogue& e) {
  const float p = __fadd_rn(__fmul_rn(__int2float_rn(t), sc), __fmul_rn(__int2float_rn(rv), rs));
  const int r = __float2int_rn(p);
  return min(max(r, e.lo - e.zp), e.hi - e.zp) + e.zp;
}

// Signed byte i (0..3) of a packed word.
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
  return static_cast<int>(static_cast<int32_t>(w << (24 - 8 * i)) >> 24);
}

__device__ __forceinline__ int32_t wrap_add(int32_t a, int32_t b) {
  return static_cast<int32_t>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
}

// Apply the epilogue to one accumulator and store it at out[idx] (element index).
__device__ __forceinline__ void epilogue_store(const Epilogue& e, void* out, size_t idx, int32_t acc, int col) {
  const int32_t t = e.bias ? wrap_add(acc, __ldg(e.bias + col)) : acc;
  if (e.out_kind == kOutS32) {
    static_cast<int32_t*>(out)[idx] = t;
  } else if (e.out_kind == kOutF32) {
    static_cast<float*>(out)[idx] = __fmul_rn(__int2float_rn(t), __ldg(e.scale + col));
  } else if (e.res) {
    static_cast<int8_t*>(out)[idx] =
        static_cast<int8_t>(requant_res(t, __ldg(e.scale + col), __ldg(e.res + idx), e.res_scale, e));
  } else {
    static_cast<int8_t*>(out)[idx] = static_cast<int8_t>(requant_one(t, __ldg(e.scale + col), e));
  }
}

}  // namespace b200q
