/*
 * b2g_oracle.c -- CPU oracle for the decode-GEMV path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, not the product.  Only tests/, the smoke entry
 * point and bench.py's CPU-baseline leg load it; the CUDA library never links
 * or calls it, and nothing in the library falls back to it.
 *
 * It restates, in plain C, the arithmetic of the reference project's hot path
 * (sudb97/Llama-3.2-3B-Instruct-gemm-optimization, files cited per function):
 *
 *   - fill_host()            kernels/gemv_fp8.cu:285-295 (srand(1234), Uniform[-0.25,0.25])
 *   - fill_x()               kernels/gemv_fp8.cu:408-413 (checkreal's x: srand(seed), same draw)
 *   - pack_e4m3()            kernels/gemv_fp8.cu:297-304 (RNE, SATFINITE, no scale)
 *   - e4m3_to_double()       kernels/gemv_fp8.cu:306-310
 *   - cpu_reference_e4m3()   kernels/gemv_fp8.cu:313-323 (fp64, k-outer, skip x==0)
 *   - cpu_reference_fp16()   kernels/gemv_fp8.cu:325-335, kernels/gemv_fp16.cu:287-297
 *   - cpu_reference_scaled() kernels/gemv_fp8.cu:470-482
 *   - per-channel / per-tensor fp16 scale + pre-divide  kernels/gemv_fp8.cu:515-543
 *   - cosine_stats()         kernels/gemv_fp8.cu:337-355
 *
 * E4M3 and binary16 rounding are written from the format definitions (OCP
 * 8-bit Floating Point Specification OFP8 rev 1.0 for E4M3 "FN": bias 7, no
 * infinities, S.1111.111 is NaN, max finite 448; IEEE 754-2008 binary16),
 * using round-to-nearest-even on an exact power-of-two grid.  Parity of these
 * encoders is pinned against the reference's own E4M3 table
 * (kernels/opt_loop/fp8_accuracy/e4m3_selftest.cu, run from the reference
 * sources) and against the reference's numpy twin
 * (kernels/opt_loop/fp8_accuracy/fp8_numpy_study.py:34-36); see tests/golden.
 *
 * Layout conventions (the same as the library's C ABI):
 *   layout 0 ("KN") : W[k*N + n], the reference's row-major [K, N]
 *   layout 1 ("NK") : W[n*K + k], nn.Linear's [out, in]
 * Activations x are [M, ldx] fp16 bit patterns (uint16_t).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_LAYOUT_KN 0
#define ORC_LAYOUT_NK 1

#define ORC_SCALE_NONE 0
#define ORC_SCALE_TENSOR_FP16 1
#define ORC_SCALE_CHANNEL_FP16 2
#define ORC_SCALE_CHANNEL_FP32 3

/* ------------------------------------------------------------------------ */
/* Rounding helpers                                                           */
/* ------------------------------------------------------------------------ */

/* Round a non-negative finite double to a binary format with `mbits` stored
 * mantissa bits and minimum normal exponent `emin` (gradual underflow below
 * it), ties to even.  a / 2^(E - mbits) is exact, so nearbyint() performs the
 * only rounding. */
static double round_to_grid(double a, int mbits, int emin) {
  if (a == 0.0) return 0.0;
  int e;
  (void)frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) */
  int E = e - 1;      /* floor(log2(a)) */
  if (E < emin) E = emin;
  const double q = ldexp(1.0, E - mbits);
  return nearbyint(a / q) * q;
}

/* binary16 bits -> float (exact). */
float orc_f16_to_f32(uint16_t h) {
  const int s = (h >> 15) & 1;
  const int e = (h >> 10) & 0x1F;
  const int m = h & 0x3FF;
  double v;
  if (e == 0) {
    v = ldexp((double)m, -24);
  } else if (e == 31) {
    v = m ? NAN : INFINITY;
  } else {
    v = ldexp(1.0 + m / 1024.0, e - 15);
  }
  return (float)(s ? -v : v);
}

/* double -> binary16 bits, round to nearest even, overflow to infinity. */
uint16_t orc_f64_to_f16(double f) {
  if (isnan(f)) return 0x7E00;
  const uint16_t sign = signbit(f) ? 0x8000 : 0;
  const double a = fabs(f);
  const double r = round_to_grid(a, 10, -14);
  if (r > 65504.0) return sign | 0x7C00;
  if (r < ldexp(1.0, -14)) return sign | (uint16_t)(r / ldexp(1.0, -24));
  int e;
  (void)frexp(r, &e);
  const int E = e - 1;
  const int m = (int)(r / ldexp(1.0, E - 10)) - 1024;
  return sign | (uint16_t)(((E + 15) << 10) | m);
}

uint16_t orc_f32_to_f16(float f) { return orc_f64_to_f16((double)f); }

/* E4M3 code -> double (exact).  kernels/gemv_fp8.cu:306-310 */
double orc_e4m3_to_f64(uint8_t b) {
  const int s = (b >> 7) & 1;
  const int e = (b >> 3) & 0xF;
  const int m = b & 7;
  double v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) {
    v = ldexp((double)m, -9);
  } else {
    v = ldexp(1.0 + m / 8.0, e - 7);
  }
  return s ? -v : v;
}

/* double -> E4M3 code, round to nearest even, saturate finite values to
 * +-448 (SATFINITE); NaN -> 0x7F. */
uint8_t orc_f64_to_e4m3(double f) {
  if (isnan(f)) return 0x7F;
  const uint8_t sign = signbit(f) ? 0x80 : 0;
  double a = fabs(f);
  if (a >= 448.0) return sign | 0x7E;
  const double r = round_to_grid(a, 3, -6);
  if (r >= 448.0) return sign | 0x7E;
  if (r < ldexp(1.0, -6)) return sign | (uint8_t)(r / ldexp(1.0, -9));
  int e;
  (void)frexp(r, &e);
  const int E = e - 1;
  const int m = (int)(r / ldexp(1.0, E - 3)) - 8;
  return sign | (uint8_t)(((E + 7) << 3) | m);
}

uint8_t orc_f32_to_e4m3(float f) { return orc_f64_to_e4m3((double)f); }

/* half -> E4M3: the half is widened exactly, so one RNE rounding happens,
 * which is what __nv_fp8_e4m3(__half) does in pack_e4m3 (gemv_fp8.cu:301). */
uint8_t orc_f16_to_e4m3(uint16_t h) { return orc_f64_to_e4m3((double)orc_f16_to_f32(h)); }

/* ------------------------------------------------------------------------ */
/* Reference input generator: kernels/gemv_fp8.cu:285-295 (same in          */
/* kernels/gemv_fp16.cu:273-285).  Uses the C library's rand() exactly as the */
/* reference does, so on the same libc the draws are identical.              */
/* ------------------------------------------------------------------------ */
void orc_fill_host_ref(uint16_t* W, size_t w_elems, uint16_t* x, int K) {
  srand(1234);
  for (size_t i = 0; i < w_elems; ++i)
    W[i] = orc_f32_to_f16(((rand() % 2001) - 1000) / 4000.0f);
  for (int i = 0; i < K; ++i)
    x[i] = orc_f32_to_f16(((rand() % 2001) - 1000) / 4000.0f);
}

void orc_fill_x_ref(uint16_t* x, int K, unsigned seed) {
  srand(seed);
  for (int i = 0; i < K; ++i)
    x[i] = orc_f32_to_f16(((rand() % 2001) - 1000) / 4000.0f);
}

/* ------------------------------------------------------------------------ */
/* Quantisation rules                                                         */
/* ------------------------------------------------------------------------ */

/* Q1, kernels/gemv_fp8.cu:297-304: q = E4M3(half w), no scale. */
void orc_pack_e4m3(const uint16_t* w16, size_t n, uint8_t* q) {
  for (size_t i = 0; i < n; ++i) q[i] = orc_f16_to_e4m3(w16[i]);
}

static inline size_t w_index(int layout, int K, int N, int k, int n) {
  return layout == ORC_LAYOUT_KN ? (size_t)k * N + n : (size_t)n * K + k;
}

/* Quantise fp16 weights to E4M3 codes under one of the four scale modes.
 *
 *  NONE           Q1 (gemv_fp8.cu:297-304); scales untouched.
 *  TENSOR_FP16    gemv_fp8.cu:517-543 with smode == kScaleTensor: one fp16
 *                 scale s = half(max(amax,1e-12f)/448) (written to scales[0]),
 *                 w' = half(float(w)/float(s)), q = E4M3(w').
 *  CHANNEL_FP16   the same with amax taken per output column n; scales[N] fp16.
 *  CHANNEL_FP32   per output channel s[n] = fp32(max(amax_n,1e-12) / 448),
 *                 q = E4M3_rn_satfinite(float(w) / s[n]) (fp32 division); the
 *                 scale/round rule stated for the FP8 benchmark configs.
 * Returns 0 on success, -1 on a bad argument.
 */
int orc_quantize_e4m3(const uint16_t* w16, int K, int N, int layout, int scale_mode,
                      uint8_t* q, void* scales) {
  if (K <= 0 || N <= 0 || (layout != 0 && layout != 1)) return -1;
  const size_t elems = (size_t)K * N;
  if (scale_mode == ORC_SCALE_NONE) {
    orc_pack_e4m3(w16, elems, q);
    return 0;
  }
  if (scale_mode < 1 || scale_mode > 3 || !scales) return -1;
  float* colmax = (float*)calloc((size_t)N, sizeof(float));
  float tmax = 0.f;
  for (int k = 0; k < K; ++k)
    for (int n = 0; n < N; ++n) {
      const float a = fabsf(orc_f16_to_f32(w16[w_index(layout, K, N, k, n)]));
      if (a > colmax[n]) colmax[n] = a;
      if (a > tmax) tmax = a;
    }
  if (scale_mode == ORC_SCALE_CHANNEL_FP32) {
    /* The 1e-12 floor is the reference's guard (gemv_fp8.cu:531) kept in
     * fp32, so an all-zero column quantises to zeros instead of 0/0. */
    float* s = (float*)scales;
    for (int n = 0; n < N; ++n) s[n] = fmaxf(colmax[n], 1e-12f) / 448.0f;
    for (int k = 0; k < K; ++k)
      for (int n = 0; n < N; ++n) {
        const size_t i = w_index(layout, K, N, k, n);
        q[i] = orc_f32_to_e4m3(orc_f16_to_f32(w16[i]) / s[n]);
      }
  } else {
    /* gemv_fp8.cu:529-539: fp16 scale, fp16 pre-divided weight, then pack. */
    uint16_t* s16 = (uint16_t*)malloc((size_t)N * sizeof(uint16_t));
    for (int n = 0; n < N; ++n) {
      const float amax = (scale_mode == ORC_SCALE_TENSOR_FP16) ? tmax : colmax[n];
      s16[n] = orc_f32_to_f16(fmaxf(amax, 1e-12f) / 448.0f);
    }
    for (int k = 0; k < K; ++k)
      for (int n = 0; n < N; ++n) {
        const size_t i = w_index(layout, K, N, k, n);
        const uint16_t wdiv = orc_f32_to_f16(orc_f16_to_f32(w16[i]) / orc_f16_to_f32(s16[n]));
        q[i] = orc_f16_to_e4m3(wdiv);
      }
    if (scale_mode == ORC_SCALE_TENSOR_FP16)
      ((uint16_t*)scales)[0] = s16[0];
    else
      memcpy(scales, s16, (size_t)N * sizeof(uint16_t));
    free(s16);
  }
  free(colmax);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* fp64 GEMV                                                                  */
/* ------------------------------------------------------------------------ */

/* y[m*N + n] = sum_k x[m,k] * deq(W[k,n]), fp64, k-outer with x==0 rows
 * skipped -- the loop of cpu_reference_e4m3 / cpu_reference_fp16
 * (gemv_fp8.cu:313-335), extended to M rows of x and either layout.
 * wtype 0: W holds fp16 bits (uint16_t); wtype 1: W holds E4M3 codes.
 * Column blocks are spread over OpenMP threads when built with -fopenmp. */
void orc_gemv_f64(const void* W, int wtype, int layout, int K, int N,
                  const uint16_t* x, int M, long ldx, double* y) {
  double lut[256];
  for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_to_f64((uint8_t)i);
  const int NB = 256;
  const int nblocks = (N + NB - 1) / NB;
#pragma omp parallel for schedule(dynamic, 1)
  for (int b = 0; b < nblocks; ++b) {
    const int n0 = b * NB;
    const int n1 = n0 + NB < N ? n0 + NB : N;
    for (int m = 0; m < M; ++m) {
      double* yr = y + (size_t)m * N;
      for (int n = n0; n < n1; ++n) yr[n] = 0.0;
      for (int k = 0; k < K; ++k) {
        const double xk = orc_f16_to_f32(x[(size_t)m * ldx + k]);
        if (xk == 0.0) continue;
        if (wtype == 1) {
          const uint8_t* w8 = (const uint8_t*)W;
          if (layout == ORC_LAYOUT_KN) {
            const uint8_t* row = w8 + (size_t)k * N;
            for (int n = n0; n < n1; ++n) yr[n] += xk * lut[row[n]];
          } else {
            for (int n = n0; n < n1; ++n) yr[n] += xk * lut[w8[(size_t)n * K + k]];
          }
        } else {
          const uint16_t* w16 = (const uint16_t*)W;
          for (int n = n0; n < n1; ++n)
            yr[n] += xk * (double)orc_f16_to_f32(w16[w_index(layout, K, N, k, n)]);
        }
      }
    }
  }
}

/* Scale epilogue as a real number: y[m,n] *= s(n) where s is fp16 or fp32
 * per-channel, or the fp16 scalar in scales[0] (cpu_reference_scaled,
 * gemv_fp8.cu:481; cast_scale_f32_to_f16_kernel, gemv_fp8.cu:164-173). */
void orc_apply_scale(double* y, int M, int N, int scale_mode, const void* scales) {
  if (scale_mode == ORC_SCALE_NONE) return;
  for (int n = 0; n < N; ++n) {
    double s;
    if (scale_mode == ORC_SCALE_CHANNEL_FP32) s = ((const float*)scales)[n];
    else if (scale_mode == ORC_SCALE_CHANNEL_FP16) s = orc_f16_to_f32(((const uint16_t*)scales)[n]);
    else s = orc_f16_to_f32(((const uint16_t*)scales)[0]);
    for (int m = 0; m < M; ++m) y[(size_t)m * N + n] *= s;
  }
}

/* Round an array of doubles to fp16 bits (RNE). */
void orc_round_f16(const double* v, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_f64_to_f16(v[i]);
}

/* cosine / max-abs / max-rel with the reference's 1e-3 denominator floor,
 * kernels/gemv_fp8.cu:337-355.  `got` are fp16 bits. */
void orc_cosine_stats(const uint16_t* got, const double* want, size_t n, double* out3) {
  double dot = 0, na = 0, nb = 0, max_abs = 0, max_rel = 0;
  for (size_t i = 0; i < n; ++i) {
    const double g = orc_f16_to_f32(got[i]);
    const double w = want[i];
    dot += g * w;
    na += g * g;
    nb += w * w;
    const double ae = fabs(g - w);
    if (ae > max_abs) max_abs = ae;
    const double den = fabs(w) > 1e-3 ? fabs(w) : 1e-3;
    if (ae / den > max_rel) max_rel = ae / den;
  }
  out3[0] = dot / (sqrt(na) * sqrt(nb));
  out3[1] = max_abs;
  out3[2] = max_rel;
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Array forms of the element conversions, for the Python wrapper. */
void orc_f16_to_e4m3_array(const uint16_t* h, size_t n, uint8_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_f16_to_e4m3(h[i]);
}
void orc_f32_to_e4m3_array(const float* f, size_t n, uint8_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_e4m3(f[i]);
}
void orc_e4m3_to_f64_array(const uint8_t* b, size_t n, double* out) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_e4m3_to_f64(b[i]);
}
void orc_f64_to_f16_array(const double* v, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_f64_to_f16(v[i]);
}
