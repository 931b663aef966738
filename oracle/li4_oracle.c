/*
 * li4_oracle.c -- CPU restatement of the reference's INT4 weight-only path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels
 * and the timed CPU baseline of bench.py; no product code path may call it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Each function restates one reference function operation by operation in
 * IEEE fp32 (SSE, no FMA contraction: build with -ffp-contract=off), with
 * fp16 storage handled through _Float16 (round-to-nearest-even):
 *   li4o_quantize    <- QuantizedLinear.quantize_tensor   llama/quantize.py:44-75
 *   li4o_dequantize  <- QuantizedLinear.dequantize_packed llama/quantize.py:78-104
 *   li4o_linear      <- QuantizedLinear.forward (v1 path: dequantize_packed +
 *                       F.linear, llama/quantize.py:143-147); the matmul sums
 *                       fp16 W times fp16 x exactly in double and rounds once to
 *                       fp16 (the reference's fp16 GEMM accumulates in fp32, so
 *                       the two differ only by accumulation rounding).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef _Float16 f16;

static inline float h2f(uint16_t h) {
  f16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static inline uint16_t f2h(float f) {
  f16 v = (f16)f; /* round to nearest even, overflow -> inf, subnormals kept */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* torch.clamp(v, 0, 15): NaN and -0.0 pass through. */
static inline float clamp_0_15(float v) {
  if (v < 0.0f) v = 0.0f;
  if (v > 15.0f) v = 15.0f;
  return v;
}

/* torch.round: round half to even (default rounding mode). */
static inline float round_even(float v) { return nearbyintf(v); }

static inline float nan_min(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return b < a ? b : a;
}

static inline float nan_max(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  return b > a ? b : a;
}

/* Load element k of row n as fp32 ("weight.float()", llama/quantize.py:62).
 * dtype: 0 = fp16, 1 = bf16, 2 = fp32. */
static inline float load_w(const void* w, int dtype, int64_t idx) {
  if (dtype == 0) return h2f(((const uint16_t*)w)[idx]);
  if (dtype == 1) return bf2f(((const uint16_t*)w)[idx]);
  return ((const float*)w)[idx];
}

/* llama/quantize.py:44-75.  Outputs contiguous packed [N, K/2], scale/zero [N, K/group]
 * (fp16 bit patterns).  Returns 0, or -1 on a bad shape. */
int li4o_quantize(const void* w, int dtype, int64_t N, int64_t K, int64_t group, int64_t stride_wn,
                  uint8_t* packed, uint16_t* scale, uint16_t* zero) {
  if (group < 2 || group % 2 || K % group) return -1;
  const int64_t G = K / group;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t g = 0; g < G; ++g) {
      const int64_t base = n * stride_wn + g * group;
      /* w_min / w_max (:64-65) */
      float mn = INFINITY, mx = -INFINITY;
      for (int64_t e = 0; e < group; ++e) {
        const float v = load_w(w, dtype, base + e);
        mn = nan_min(mn, v);
        mx = nan_max(mx, v);
      }
      /* scale = (max - min) / 15 ; 0 -> 1 (:67-68) */
      float s = (mx - mn) / 15.0f;
      if (s == 0.0f) s = 1.0f;
      /* zero_point = round(-min / scale).clamp(0, 15) (:69) */
      const float zp = clamp_0_15(round_even(-mn / s));
      /* q = round(w / scale + zero_point).clamp(0, 15), packed even | odd << 4 (:71-73) */
      for (int64_t j = 0; j < group / 2; ++j) {
        const float t0 = load_w(w, dtype, base + 2 * j) / s;
        const float t1 = load_w(w, dtype, base + 2 * j + 1) / s;
        const float q0 = clamp_0_15(round_even(t0 + zp));
        const float q1 = clamp_0_15(round_even(t1 + zp));
        packed[n * (K / 2) + g * (group / 2) + j] = (uint8_t)((unsigned)q0 | ((unsigned)q1 << 4));
      }
      /* scale.half(), zero_point.half() (:75) */
      scale[n * G + g] = f2h(s);
      zero[n * G + g] = f2h(zp);
    }
  }
  return 0;
}

/* One dequantized weight: fp32 (q - zero) * scale, then .half() (:101-104). */
static inline uint16_t dequant_one(unsigned q, float z, float s) {
  const float d = (float)q - z;
  return f2h(d * s);
}

/* llama/quantize.py:78-104.  w16 [N, K] fp16 bit patterns, row stride stride_wn. */
int li4o_dequantize(const uint8_t* packed, const uint16_t* scale, const uint16_t* zero, int64_t N, int64_t K,
                    int64_t group, int64_t stride_pn, int64_t stride_sn, int64_t stride_wn, uint16_t* w16) {
  if (group < 2 || group % 2 || K % group) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t k = 0; k < K; ++k) {
      const uint8_t b = packed[n * stride_pn + k / 2];
      const unsigned q = (k & 1) ? (unsigned)(b >> 4) : (unsigned)(b & 0x0F); /* :95-99 */
      const int64_t g = k / group;
      w16[n * stride_wn + k] = dequant_one(q, h2f(zero[n * stride_sn + g]), h2f(scale[n * stride_sn + g]));
    }
  }
  return 0;
}

/* QuantizedLinear.forward, v1 path (llama/quantize.py:143-147):
 *   y[m, n] = fp16( sum_k W16[n, k] * x[m, k] ),  W16 = dequantize_packed(...)
 * x [M, K] fp16 (row stride stride_xm), y [M, N] fp16 (row stride stride_ym),
 * y32 (optional) [M, N] fp32 copy of the unrounded sums.  Each row of W is
 * dequantized exactly as li4o_dequantize does; the dot product is accumulated
 * in double (every fp16 x fp16 product is exact in double) and rounded once. */
int li4o_linear(const uint16_t* x, const uint8_t* packed, const uint16_t* scale, const uint16_t* zero, int64_t M,
                int64_t N, int64_t K, int64_t group, int64_t stride_xm, int64_t stride_pn, int64_t stride_sn,
                int64_t stride_ym, uint16_t* y, float* y32) {
  if (group < 2 || group % 2 || K % group || M < 0 || N < 0) return -1;
  float* xf = (float*)malloc((size_t)(M > 0 ? M : 1) * (size_t)(K > 0 ? K : 1) * sizeof(float));
  if (!xf) return -2;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) xf[m * K + k] = h2f(x[m * stride_xm + k]);
  int failed = 0;
#pragma omp parallel reduction(| : failed)
  {
    float* wrow = (float*)malloc((size_t)(K > 0 ? K : 1) * sizeof(float));
    if (!wrow) failed = 1;
#pragma omp for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
      if (!wrow) continue;
      const uint8_t* prow = packed + n * stride_pn;
      for (int64_t g = 0; g < K / group; ++g) {
        const float z = h2f(zero[n * stride_sn + g]);
        const float s = h2f(scale[n * stride_sn + g]);
        for (int64_t k = g * group; k < (g + 1) * group; k += 2) {
          const uint8_t b = prow[k / 2];
          wrow[k] = h2f(dequant_one((unsigned)(b & 0x0F), z, s));
          wrow[k + 1] = h2f(dequant_one((unsigned)(b >> 4), z, s));
        }
      }
      for (int64_t m = 0; m < M; ++m) {
        /* four partial sums in double: every product is exact, the sums carry 53 bits */
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        const float* xr = xf + m * K;
        int64_t k = 0;
        for (; k + 4 <= K; k += 4) {
          a0 += (double)wrow[k] * (double)xr[k];
          a1 += (double)wrow[k + 1] * (double)xr[k + 1];
          a2 += (double)wrow[k + 2] * (double)xr[k + 2];
          a3 += (double)wrow[k + 3] * (double)xr[k + 3];
        }
        for (; k < K; ++k) a0 += (double)wrow[k] * (double)xr[k];
        const double acc = (a0 + a1) + (a2 + a3);
        if (y) {
          f16 h = (f16)acc; /* one rounding, double -> fp16 */
          memcpy(&y[m * stride_ym + n], &h, 2);
        }
        if (y32) y32[m * N + n] = (float)acc;
      }
    }
    free(wrow);
  }
  free(xf);
  return failed ? -2 : 0;
}

/* Threads the OpenMP runtime will use (1 without OpenMP). */
int li4o_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void li4o_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
