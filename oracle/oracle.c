/*
 * CPU oracle for the int8 / quantized-int32 convolution and batched-GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/, the
 * smoke() entry of __graft_entry__.py and the cpu_baseline leg of bench.py
 * may load it.  Nothing on the product path links or calls it.
 *
 * It is a plain-C restatement of the reference algorithms:
 *   - quantized conv fprop, int32 accumulators:
 *       NikitaYak02/my_own_cnn src/cpu_ref.cpp:36-72 (regular) and :74-112 (blocked),
 *       zero points from src/nnalgebra_quantization.h:56-69,
 *       output shape / validation from src/conv_types.h:125-169;
 *   - int32 batched GEMM with four transpose modes: bmm.h:9-29, bmm.cu:155-246
 *     (int32 wrap-around accumulate; done here in uint32 to avoid C signed-overflow UB);
 *   - the requantization epilogue, which the reference does not have (new semantics):
 *       t = acc + bias[k]            (int32, wrapping)
 *       f = (float)t                 (round to nearest even)
 *       p = f * scale[k]             (one fp32 multiply, no contraction)
 *       r = rint_sat(p)              (round half to even, saturated to int32, NaN -> 0)
 *       q = clamp(r, lo - zp, hi - zp) + zp
 *     and the dequantized fp32 output  y = (float)(acc + bias[k]) * scale[k];
 *     with a fused residual add, p gains + (float)res * res_scale before rounding;
 *   - int8 max pool and global average pool (new; the int8 network stacks between convs).
 *   - a counter-based splitmix64 generator that the CUDA library implements
 *     identically, so any slice of a synthetic tensor can be regenerated here.
 *
 * Built with -ffp-contract=off so that no multiply-add is fused.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_EINVAL 1

/* ---------------------------------------------------------------- shapes */

/* conv_types.h:125-146 (infer_conv_shape): same checks, same formula. */
int orc_conv_out_shape(int h, int w, int c, int r, int s, int k, int pad_h, int pad_w, int stride_h,
                       int stride_w, int dil_h, int dil_w, int groups, int* ho, int* wo) {
  if (groups <= 0) return ORC_EINVAL;
  if (c % groups != 0) return ORC_EINVAL;
  if (k % groups != 0) return ORC_EINVAL;
  int hn = h + 2 * pad_h - dil_h * (r - 1) - 1;
  int wn = w + 2 * pad_w - dil_w * (s - 1) - 1;
  if (hn < 0 || wn < 0) return ORC_EINVAL;
  if (stride_h <= 0 || stride_w <= 0) return ORC_EINVAL;
  *ho = hn / stride_h + 1;
  *wo = wn / stride_w + 1;
  if (*ho <= 0 || *wo <= 0) return ORC_EINVAL;
  return ORC_OK;
}

typedef struct {
  int n, h, w, c, r, s, k;
  int pad_h, pad_w, stride_h, stride_w, dil_h, dil_w, groups;
  int by, bx; /* block grid; 1,1 for a regular conv */
} orc_conv_t;

/*
 * Quantized conv, int32 accumulators (cpu_ref.cpp:36-72 / :74-112).
 * x: NHWC codes as float, w: KRSC (or K,By,Bx,R,S,C for blocked) codes as float,
 * zp_in: per-image input zero point, zp_f: filter zero point.
 * Padding taps are skipped, which equals a centred value of 0.
 * Images [n_begin, n_end) are computed; y is the full NHWC output.
 */
static void conv_qi32_range(const orc_conv_t* p, const float* x, const float* w, int32_t* y,
                            const int32_t* zp_in, int32_t zp_f, int ho_n, int wo_n, int n_begin,
                            int n_end) {
  const int cg = p->c / p->groups, kg = p->k / p->groups;
  const int bho = ho_n / p->by, bwo = wo_n / p->bx;
  for (int n = n_begin; n < n_end; ++n) {
    const int32_t zx = zp_in[n];
    for (int ho = 0; ho < ho_n; ++ho) {
      const int by = ho / bho;
      for (int wo = 0; wo < wo_n; ++wo) {
        const int bx = wo / bwo;
        for (int g = 0; g < p->groups; ++g) {
          for (int ko = 0; ko < kg; ++ko) {
            const int kk = g * kg + ko;
            uint32_t acc = 0;
            for (int rr = 0; rr < p->r; ++rr) {
              const int hi = ho * p->stride_h - p->pad_h + rr * p->dil_h;
              if (hi < 0 || hi >= p->h) continue;
              for (int ss = 0; ss < p->s; ++ss) {
                const int wi = wo * p->stride_w - p->pad_w + ss * p->dil_w;
                if (wi < 0 || wi >= p->w) continue;
                const float* xp = x + (((size_t)n * p->h + hi) * p->w + wi) * p->c + (size_t)g * cg;
                const float* wp =
                    w + (((((size_t)kk * p->by + by) * p->bx + bx) * p->r + rr) * p->s + ss) * cg;
                for (int ci = 0; ci < cg; ++ci) {
                  const int32_t xv = (int32_t)xp[ci] - zx;
                  const int32_t wv = (int32_t)wp[ci] - zp_f;
                  acc += (uint32_t)xv * (uint32_t)wv;
                }
              }
            }
            y[(((size_t)n * ho_n + ho) * wo_n + wo) * p->k + kk] = (int32_t)acc;
          }
        }
      }
    }
  }
}

int orc_conv_qi32(const orc_conv_t* p, const float* x, const float* w, int32_t* y,
                  const int32_t* zp_in, int32_t zp_f) {
  int ho, wo;
  if (orc_conv_out_shape(p->h, p->w, p->c, p->r, p->s, p->k, p->pad_h, p->pad_w, p->stride_h,
                         p->stride_w, p->dil_h, p->dil_w, p->groups, &ho, &wo))
    return ORC_EINVAL;
  /* conv_types.h:148-169 (infer_block_conv_shape) */
  if (p->by <= 0 || p->bx <= 0) return ORC_EINVAL;
  if (ho % p->by || wo % p->bx) return ORC_EINVAL;
  conv_qi32_range(p, x, w, y, zp_in, zp_f, ho, wo, 0, p->n);
  return ORC_OK;
}

/*
 * Same conv on int8 tensors with zero points 0 -- the int32 accumulators that
 * the int8 tensor-core kernel must reproduce bit-exactly.  (Converting int8 to
 * float codes and calling the path above gives the same numbers; this variant
 * only avoids the 4x memory of float codes.)
 */
typedef struct {
  const orc_conv_t* p;
  const int8_t* x;
  const int8_t* w;
  int32_t* y;
  int ho, wo, n0, n1;
} s8_job_t;

static void conv_s8_range(const orc_conv_t* p, const int8_t* x, const int8_t* w, int32_t* y,
                          int ho_n, int wo_n, int n_begin, int n_end) {
  const int cg = p->c / p->groups, kg = p->k / p->groups;
  const int bho = ho_n / p->by, bwo = wo_n / p->bx;
  for (int n = n_begin; n < n_end; ++n)
    for (int ho = 0; ho < ho_n; ++ho) {
      const int by = ho / bho;
      for (int wo = 0; wo < wo_n; ++wo) {
        const int bx = wo / bwo;
        int32_t* yp = y + (((size_t)n * ho_n + ho) * wo_n + wo) * p->k;
        for (int kk = 0; kk < p->k; ++kk) yp[kk] = 0;
        for (int rr = 0; rr < p->r; ++rr) {
          const int hi = ho * p->stride_h - p->pad_h + rr * p->dil_h;
          if (hi < 0 || hi >= p->h) continue;
          for (int ss = 0; ss < p->s; ++ss) {
            const int wi = wo * p->stride_w - p->pad_w + ss * p->dil_w;
            if (wi < 0 || wi >= p->w) continue;
            const int8_t* xp = x + (((size_t)n * p->h + hi) * p->w + wi) * p->c;
            for (int g = 0; g < p->groups; ++g)
              for (int ko = 0; ko < kg; ++ko) {
                const int kk = g * kg + ko;
                const int8_t* wp =
                    w + (((((size_t)kk * p->by + by) * p->bx + bx) * p->r + rr) * p->s + ss) * cg;
                const int8_t* xg = xp + (size_t)g * cg;
                int32_t acc = 0; /* |partial| <= cg*127*128, fits for cg < 131072 */
                for (int ci = 0; ci < cg; ++ci) acc += (int32_t)xg[ci] * (int32_t)wp[ci];
                yp[kk] = (int32_t)((uint32_t)yp[kk] + (uint32_t)acc);
              }
          }
        }
      }
    }
}

static void* s8_worker(void* arg) {
  s8_job_t* j = (s8_job_t*)arg;
  conv_s8_range(j->p, j->x, j->w, j->y, j->ho, j->wo, j->n0, j->n1);
  return NULL;
}

/* Images are independent, so a batch split over threads is exact. */
int orc_conv_s8(const orc_conv_t* p, const int8_t* x, const int8_t* w, int32_t* y, int threads) {
  int ho, wo;
  if (orc_conv_out_shape(p->h, p->w, p->c, p->r, p->s, p->k, p->pad_h, p->pad_w, p->stride_h,
                         p->stride_w, p->dil_h, p->dil_w, p->groups, &ho, &wo))
    return ORC_EINVAL;
  if (p->by <= 0 || p->bx <= 0 || ho % p->by || wo % p->bx) return ORC_EINVAL;
  if (threads <= 1 || p->n <= 1) {
    conv_s8_range(p, x, w, y, ho, wo, 0, p->n);
    return ORC_OK;
  }
  if (threads > p->n) threads = p->n;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  s8_job_t* jobs = (s8_job_t*)malloc(sizeof(s8_job_t) * threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t].p = p; jobs[t].x = x; jobs[t].w = w; jobs[t].y = y;
    jobs[t].ho = ho; jobs[t].wo = wo;
    jobs[t].n0 = (int)((long long)p->n * t / threads);
    jobs[t].n1 = (int)((long long)p->n * (t + 1) / threads);
    pthread_create(&th[t], NULL, s8_worker, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
  return ORC_OK;
}

/* ------------------------------------------------------------- epilogue */

/* float -> int32, round half to even, saturating, NaN -> 0 (the PTX cvt.rni.s32.f32 rule). */
static int32_t rint_sat(float p) {
  if (p != p) return 0;
  if (p >= 2147483648.0f) return INT32_MAX;
  if (p < -2147483648.0f) return INT32_MIN;
  return (int32_t)nearbyintf(p);
}

/* Requantize int32 accumulators [rows][k] to int8 codes.  bias may be NULL (0). */
void orc_requant_s8(const int32_t* acc, size_t rows, int k, const int32_t* bias, const float* scale,
                    int zp, int lo, int hi, int8_t* out) {
  for (size_t i = 0; i < rows; ++i)
    for (int j = 0; j < k; ++j) {
      const uint32_t t = (uint32_t)acc[i * k + j] + (uint32_t)(bias ? bias[j] : 0);
      const float f = (float)(int32_t)t;
      const float pr = f * scale[j];
      int32_t r = rint_sat(pr);
      if (r < lo - zp) r = lo - zp;
      if (r > hi - zp) r = hi - zp;
      out[i * k + j] = (int8_t)(r + zp);
    }
}

/* Requantize with a fused residual add (the int8 residual res has the accumulators' layout):
 *   p = (float)(acc + bias) * scale[k] + (float)res * res_scale   (each step one IEEE operation)
 *   q = clamp(rint_sat(p), lo - zp, hi - zp) + zp */
void orc_requant_res_s8(const int32_t* acc, size_t rows, int k, const int32_t* bias, const float* scale,
                        const int8_t* res, float res_scale, int zp, int lo, int hi, int8_t* out) {
  for (size_t i = 0; i < rows; ++i)
    for (int j = 0; j < k; ++j) {
      const uint32_t t = (uint32_t)acc[i * k + j] + (uint32_t)(bias ? bias[j] : 0);
      const float pr = (float)(int32_t)t * scale[j];
      const float rr = (float)res[i * k + j] * res_scale;
      const float p = pr + rr;
      int32_t r = rint_sat(p);
      if (r < lo - zp) r = lo - zp;
      if (r > hi - zp) r = hi - zp;
      out[i * k + j] = (int8_t)(r + zp);
    }
}

/* Max pool, NHWC int8, R x S window, stride / padding; padded positions take no part. */
int orc_maxpool_s8(const int8_t* x, int8_t* y, int n, int h, int w, int c, int r, int s, int stride_h,
                   int stride_w, int pad_h, int pad_w) {
  const int ho = (h + 2 * pad_h - r) / stride_h + 1, wo = (w + 2 * pad_w - s) / stride_w + 1;
  if (ho <= 0 || wo <= 0) return ORC_EINVAL;
  for (int b = 0; b < n; ++b)
    for (int oh = 0; oh < ho; ++oh)
      for (int ow = 0; ow < wo; ++ow)
        for (int ch = 0; ch < c; ++ch) {
          int m = -128;
          for (int i = 0; i < r; ++i)
            for (int j = 0; j < s; ++j) {
              const int ih = oh * stride_h - pad_h + i, iw = ow * stride_w - pad_w + j;
              if (ih < 0 || ih >= h || iw < 0 || iw >= w) continue;
              const int v = x[(((size_t)b * h + ih) * w + iw) * c + ch];
              if (v > m) m = v;
            }
          y[(((size_t)b * ho + oh) * wo + ow) * c + ch] = (int8_t)m;
        }
  return ORC_OK;
}

/* Global average pool, NHWC int8 -> [n][c]: q = clamp(rint_sat((float)sum / (float)(h*w)), -128, 127)
 * (sum exact in int32; one IEEE division). */
void orc_global_avgpool_s8(const int8_t* x, int8_t* y, int n, int h, int w, int c) {
  const float cnt = (float)(h * w);
  for (int b = 0; b < n; ++b)
    for (int ch = 0; ch < c; ++ch) {
      int32_t sum = 0;
      for (int i = 0; i < h * w; ++i) sum += x[((size_t)b * h * w + i) * c + ch];
      int32_t q = rint_sat((float)sum / cnt);
      if (q < -128) q = -128;
      if (q > 127) q = 127;
      y[(size_t)b * c + ch] = (int8_t)q;
    }
}

void orc_dequant_f32(const int32_t* acc, size_t rows, int k, const int32_t* bias,
                     const float* scale, float* out) {
  for (size_t i = 0; i < rows; ++i)
    for (int j = 0; j < k; ++j) {
      const uint32_t t = (uint32_t)acc[i * k + j] + (uint32_t)(bias ? bias[j] : 0);
      out[i * k + j] = (float)(int32_t)t * scale[j];
    }
}

/* ----------------------------------------------------------------- bmm */

/* bmm.h:9-29 layout conventions; int32 wrap-around like bmm.cu:218-229. */
void orc_bmm_i32(const int32_t* A, const int32_t* B, int32_t* C, int batch, int M, int N, int K,
                 int ta, int tb) {
  for (int b = 0; b < batch; ++b) {
    const int32_t* Ab = A + (size_t)b * M * K;
    const int32_t* Bb = B + (size_t)b * K * N;
    int32_t* Cb = C + (size_t)b * M * N;
    for (int m = 0; m < M; ++m)
      for (int n = 0; n < N; ++n) {
        uint32_t acc = 0;
        for (int kk = 0; kk < K; ++kk) {
          const int32_t a = ta ? Ab[(size_t)kk * M + m] : Ab[(size_t)m * K + kk];
          const int32_t v = tb ? Bb[(size_t)n * K + kk] : Bb[(size_t)kk * N + n];
          acc += (uint32_t)a * (uint32_t)v;
        }
        Cb[(size_t)m * N + n] = (int32_t)acc;
      }
  }
}

typedef struct {
  const int8_t *A, *B;
  int32_t* C;
  int M, N, K, ta, tb, b0, b1;
} bmm_job_t;

static void bmm_s8_range(const bmm_job_t* j) {
  int32_t* col = (int32_t*)malloc(sizeof(int32_t) * (size_t)j->K);
  for (int b = j->b0; b < j->b1; ++b) {
    const int8_t* Ab = j->A + (size_t)b * j->M * j->K;
    const int8_t* Bb = j->B + (size_t)b * j->K * j->N;
    int32_t* Cb = j->C + (size_t)b * j->M * j->N;
    for (int n = 0; n < j->N; ++n) {
      for (int kk = 0; kk < j->K; ++kk)
        col[kk] = j->tb ? Bb[(size_t)n * j->K + kk] : Bb[(size_t)kk * j->N + n];
      for (int m = 0; m < j->M; ++m) {
        int32_t acc = 0; /* |acc| <= K*127*128 fits for K < 131072 */
        if (!j->ta) {
          const int8_t* ar = Ab + (size_t)m * j->K;
          for (int kk = 0; kk < j->K; ++kk) acc += (int32_t)ar[kk] * col[kk];
        } else {
          for (int kk = 0; kk < j->K; ++kk) acc += (int32_t)Ab[(size_t)kk * j->M + m] * col[kk];
        }
        Cb[(size_t)m * j->N + n] = acc;
      }
    }
  }
  free(col);
}

static void* bmm_worker(void* arg) {
  bmm_s8_range((bmm_job_t*)arg);
  return NULL;
}

/* int8 batched GEMM with int32 outputs; batch items split over threads. */
void orc_bmm_s8(const int8_t* A, const int8_t* B, int32_t* C, int batch, int M, int N, int K,
                int ta, int tb, int threads) {
  if (threads < 1) threads = 1;
  if (threads > batch) threads = batch;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  bmm_job_t* jobs = (bmm_job_t*)malloc(sizeof(bmm_job_t) * threads);
  for (int t = 0; t < threads; ++t) {
    bmm_job_t j = {A, B, C, M, N, K, ta, tb, (int)((long long)batch * t / threads),
                   (int)((long long)batch * (t + 1) / threads)};
    jobs[t] = j;
    pthread_create(&th[t], NULL, bmm_worker, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}

/* ----------------------------------------------------------- generator */

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Stream key for (seed, tensor id); element i draws mix64(key + (i+1)*golden). */
uint64_t orc_stream_key(uint64_t seed, uint64_t tensor_id) {
  return mix64(seed * 0x9E3779B97F4A7C15ull ^ mix64(tensor_id + 0x632BE59BD9B4E019ull));
}

static inline uint64_t draw(uint64_t key, uint64_t i) {
  return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull);
}

/* Uniform integers in [lo, hi] for elements [offset, offset+count). */
void orc_fill_s8_uniform(uint64_t seed, uint64_t tensor_id, int lo, int hi, size_t offset,
                         size_t count, int8_t* out) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
  const uint64_t span = (uint64_t)(hi - lo + 1);
  for (size_t i = 0; i < count; ++i)
    out[i] = (int8_t)(lo + (int)(((draw(key, offset + i) >> 32) * span) >> 32));
}

void orc_fill_i32_uniform(uint64_t seed, uint64_t tensor_id, int32_t lo, int32_t hi, size_t offset,
                          size_t count, int32_t* out) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
  const uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo + 1);
  for (size_t i = 0; i < count; ++i)
    out[i] = (int32_t)((int64_t)lo + (int64_t)(((draw(key, offset + i) >> 32) * span) >> 32));
}

/* Codes from a 65536-entry quantile table (normal / half-normal draws, exact on any device). */
void orc_fill_s8_table(uint64_t seed, uint64_t tensor_id, const int8_t* table, size_t offset,
                       size_t count, int8_t* out) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
  for (size_t i = 0; i < count; ++i) out[i] = table[draw(key, offset + i) >> 48];
}

/* Uniform floats in [lo, hi): lo + u*(hi-lo) with u = top 24 bits * 2^-24, fp32 ops. */
void orc_fill_f32_uniform(uint64_t seed, uint64_t tensor_id, float lo, float hi, size_t offset,
                          size_t count, float* out) {
  const uint64_t key = orc_stream_key(seed, tensor_id);
  const float span = hi - lo;
  for (size_t i = 0; i < count; ++i) {
    const float u = (float)(draw(key, offset + i) >> 40) * (1.0f / 16777216.0f);
    out[i] = lo + u * span;
  }
}
