/*
 * CPU oracle for the GEMM path — TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load this library; the product never calls it.
 *
 * What it restates. The reference (govindansriram/maia, kernel_lib) ships the descriptor encoders
 * for a Blackwell GEMM but no GEMM and no CPU GEMM of its own; its GEMM contract is the one
 * the descriptors encode: C = A . B^T with A [M,K] and B [N,K] both K-major
 * (kernel_lib/include/kl/layout/umma_desc.hpp:49-58, a_major = b_major = K;
 * kernel_lib/include/kl/layout/smem_tile.hpp:44-47, "MMA operands are (M or N, K), so they are
 * K-major"), bf16 or fp8 inputs, fp32 accumulation. GEMM parity is therefore unpinned against the
 * reference: there is no reference GEMM output to pin to. The tests pin this file instead against
 * numpy float64 matmul on the same decoded inputs.
 *
 *   kl_oracle_gemm_f64   fp64 accumulation over the decoded inputs, times `scale`: the result the GPU
 *                        tests compare against.
 *   kl_oracle_gemm_f32   fp32 accumulation, cache-blocked, all host threads: the timed CPU
 *                        baseline (the "CPU reference GEMM" of the benchmark's smallest config).
 *   kl_oracle_decode     element decoders (bf16, f16, e4m3, e5m2), exposed so tests can check
 *                        them.
 *   kl_oracle_gemm_mx_f64 / _f32   the same with MX block scaling (OCP Microscaling Formats v1.0):
 *                        element k of row r of A is multiplied by 2^(sfa[r][k/32] - 127) (UE8M0,
 *                        one scale per 32 consecutive K-elements; 255 is NaN), likewise for B.
 *   kl_oracle_gemm_bs_f64 / _f32   block scaling with `vec` elements per scale and the scale
 *                        format given: UE8M0 as above, or UE4M3 (NVFP4: an e4m3 byte read as a
 *                        magnitude, one scale per 16 K-elements).
 *
 * Element decoding follows the formats' definitions: bf16 is the top half of an IEEE binary32;
 * f16 is IEEE binary16 (1 sign, 5 exponent bits with bias 15, 10 mantissa bits); e4m3 (OCP FP8,
 * "fn" variant) has 1 sign, 4 exponent (bias 7), 3 mantissa bits, no infinities, and S.1111.111 is
 * NaN; e5m2 (OCP FP8) has 1 sign, 5 exponent (bias 15), 2 mantissa bits, with IEEE infinities and
 * NaNs at exponent 31; e2m1 (OCP fp4) has 1 sign, 2 exponent (bias 1), 1 mantissa bit, no
 * infinities or NaNs (values 0, 0.5, 1, 1.5, 2, 3, 4, 6), stored two per byte with the first
 * element in the low nibble. e3m2 and e2m3 (OCP fp6) have 1 sign, 3 exponent (bias 3) and 2
 * mantissa bits, or 2 exponent (bias 1) and 3 mantissa bits, no infinities or NaNs (largest 28 and
 * 7.5), packed four to three bytes: element i of a row at bits [6i, 6i + 6) of its bytes, least
 * significant bit first. Type codes follow the library's kl_dtype: bf16 0, f16 1, e4m3 2, e5m2 3,
 * e2m1 8, e3m2 11, e2m3 12.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KL_ORACLE_BF16 0
#define KL_ORACLE_F16 1
#define KL_ORACLE_E4M3 2
#define KL_ORACLE_E5M2 3
#define KL_ORACLE_E2M1 8 /* two per byte, the first in the low nibble */
#define KL_ORACLE_E3M2 11 /* four per three bytes, least significant bits first */
#define KL_ORACLE_E2M3 12

static int elem_size(int t) { return (t == KL_ORACLE_BF16 || t == KL_ORACLE_F16) ? 2 : 1; }

/* Bytes of `count` elements of type t (packed e2m1: two per byte, count even; packed fp6: four
 * per three bytes, count a multiple of 4). */
static size_t bytes_of(int t, int64_t count) {
  if (t == KL_ORACLE_E2M1) return (size_t)(count / 2);
  if (t == KL_ORACLE_E3M2 || t == KL_ORACLE_E2M3) return (size_t)(count / 4 * 3);
  return (size_t)count * (size_t)elem_size(t);
}

/* A sign-magnitude minifloat with `eb` exponent bits (bias 2^(eb-1) - 1), `mb` mantissa bits and
 * no special values: fp6 e3m2 (3, 2) and e2m3 (2, 3). */
static double decode_finite(uint32_t v, int eb, int mb) {
  const int sign = (v >> (eb + mb)) & 1;
  const int exp = (v >> mb) & ((1 << eb) - 1);
  const uint32_t man = v & ((1u << mb) - 1);
  const int bias = (1 << (eb - 1)) - 1;
  const double x = exp == 0 ? ldexp((double)man, 1 - bias - mb) : ldexp((double)((1u << mb) | man), exp - bias - mb);
  return sign ? -x : x;
}

static double decode_bf16(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, sizeof f);
  return (double)f;
}

static double decode_e4m3(uint8_t v) {
  const int sign = (v >> 7) & 1;
  const int exp = (v >> 3) & 0xF;
  const int man = v & 0x7;
  double x;
  if (exp == 0xF && man == 0x7) return NAN;
  if (exp == 0)
    x = ldexp((double)man / 8.0, -6); /* subnormal: 0.mmm * 2^(1-7) */
  else
    x = ldexp(1.0 + (double)man / 8.0, exp - 7);
  return sign ? -x : x;
}

/* IEEE-style binary format with `eb` exponent bits (bias 2^(eb-1) - 1) and `mb` mantissa bits:
 * f16 (5, 10) and e5m2 (5, 2). The all-ones exponent holds infinities and NaNs. */
static double decode_ieee(uint32_t v, int eb, int mb) {
  const int sign = (v >> (eb + mb)) & 1;
  const int exp = (v >> mb) & ((1 << eb) - 1);
  const uint32_t man = v & ((1u << mb) - 1);
  const int bias = (1 << (eb - 1)) - 1;
  double x;
  if (exp == (1 << eb) - 1)
    x = man ? NAN : INFINITY;
  else if (exp == 0)
    x = ldexp((double)man, 1 - bias - mb); /* subnormal: 0.m * 2^(1-bias) */
  else
    x = ldexp((double)((1u << mb) | man), exp - bias - mb);
  return sign ? -x : x;
}

/* Decode `n` elements of type `t` (KL_ORACLE_*) to double. */
void kl_oracle_decode(int t, const void* src, int64_t n, double* dst) {
  if (t == KL_ORACLE_BF16) {
    const uint16_t* s = (const uint16_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = decode_bf16(s[i]);
  } else if (t == KL_ORACLE_F16) {
    const uint16_t* s = (const uint16_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = decode_ieee(s[i], 5, 10);
  } else if (t == KL_ORACLE_E5M2) {
    const uint8_t* s = (const uint8_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = decode_ieee(s[i], 5, 2);
  } else if (t == KL_ORACLE_E3M2 || t == KL_ORACLE_E2M3) {
    const int eb = t == KL_ORACLE_E3M2 ? 3 : 2;
    const uint8_t* s = (const uint8_t*)src;
    for (int64_t i = 0; i < n; ++i) {
      const int64_t bit = 6 * i, byte = bit >> 3;
      const int shift = (int)(bit & 7);
      uint32_t w = s[byte];
      if (shift > 2) w |= (uint32_t)s[byte + 1] << 8; /* the element spills into the next byte */
      dst[i] = decode_finite((w >> shift) & 63u, eb, 5 - eb);
    }
  } else if (t == KL_ORACLE_E2M1) {
    double table[16];
    for (uint32_t v = 0; v < 16; ++v) {
      const double mag = (v & 6) == 0 ? 0.5 * (v & 1) : ldexp(1.0 + 0.5 * (v & 1), (int)((v >> 1) & 3) - 1);
      table[v] = (v & 8) ? -mag : mag;
    }
    const uint8_t* s = (const uint8_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = table[(s[i / 2] >> (4 * (i & 1))) & 0xF];
  } else {
    const uint8_t* s = (const uint8_t*)src;
    for (int64_t i = 0; i < n; ++i) dst[i] = decode_e4m3(s[i]);
  }
}

typedef struct {
  int t;
  const void* a;
  int64_t lda;
  const void* b;
  int64_t ldb;
  int64_t m, n, k;
  double scale;
  void* c;
  int64_t ldc;
  int64_t row_begin, row_end;
  const double* bdec; /* decoded B, n x k (f64 path) */
  const float* bdecf; /* decoded B, n x k (f32 path) */
  const uint8_t* sfa; /* optional block scales of A, row-major [m][ldsfa] */
  int64_t ldsfa;
  int vec;            /* K-elements per scale */
  int sf_ue4m3;       /* scale format: 0 = UE8M0, 1 = UE4M3 */
} job_t;

static double e8m0_table[256];
static pthread_once_t e8m0_once = PTHREAD_ONCE_INIT;
static void e8m0_init(void) {
  for (int s = 0; s < 256; ++s) e8m0_table[s] = s == 255 ? NAN : ldexp(1.0, s - 127);
}
static double e8m0(uint8_t s) { return e8m0_table[s]; }

static double ue4m3(uint8_t s) { return decode_e4m3((uint8_t)(s & 0x7F)); }

/* Decode row `r` of a matrix (k elements) and apply its block scales when `sf` is given. */
static void decode_row(int t, const void* base, int64_t ld, int64_t r, int64_t k, const uint8_t* sf, int64_t ldsf,
                       int vec, int sf_ue4m3, double* out) {
  kl_oracle_decode(t, (const char*)base + bytes_of(t, r * ld), k, out);
  pthread_once(&e8m0_once, e8m0_init);
  if (sf)
    for (int64_t kk = 0; kk < k; ++kk) {
      const uint8_t v = sf[r * ldsf + kk / vec];
      out[kk] *= sf_ue4m3 ? ue4m3(v) : e8m0(v);
    }
}

static void* f64_rows(void* arg) {
  job_t* j = (job_t*)arg;
  double* arow = (double*)malloc(sizeof(double) * (size_t)j->k);
  double* c = (double*)j->c;
  for (int64_t i = j->row_begin; i < j->row_end; ++i) {
    decode_row(j->t, j->a, j->lda, i, j->k, j->sfa, j->ldsfa, j->vec, j->sf_ue4m3, arow);
    for (int64_t col = 0; col < j->n; ++col) {
      const double* brow = j->bdec + (size_t)col * (size_t)j->k;
      double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
      int64_t kk = 0;
      for (; kk + 4 <= j->k; kk += 4) {
        s0 += arow[kk] * brow[kk];
        s1 += arow[kk + 1] * brow[kk + 1];
        s2 += arow[kk + 2] * brow[kk + 2];
        s3 += arow[kk + 3] * brow[kk + 3];
      }
      for (; kk < j->k; ++kk) s0 += arow[kk] * brow[kk];
      c[(size_t)(i * j->ldc + col)] = ((s0 + s1) + (s2 + s3)) * j->scale;
    }
  }
  free(arow);
  return NULL;
}

static int clamp_threads(int threads, int64_t rows) {
  if (threads < 1) threads = 1;
  if (threads > 512) threads = 512;
  if (rows < threads) threads = (int)(rows > 0 ? rows : 1);
  return threads;
}

/* c[i*ldc + j] = scale * sum_k A[i,k] * B[j,k] in double, for rows [0, m); with sfa / sfb (MX
 * scales, row-major, row pitch ldsfa / ldsfb) each element is scaled first. Returns 0 on success. */
int kl_oracle_gemm_bs_f64(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                          int64_t k, const uint8_t* sfa, int64_t ldsfa, const uint8_t* sfb, int64_t ldsfb, int vec,
                          int sf_ue4m3, double scale, double* c, int64_t ldc, int threads) {
  if (vec <= 0) return 2;
  double* bdec = (double*)malloc(sizeof(double) * (size_t)n * (size_t)(k > 0 ? k : 1));
  if (!bdec) return 1;
  for (int64_t r = 0; r < n; ++r) decode_row(t, b, ldb, r, k, sfb, ldsfb, vec, sf_ue4m3, bdec + r * k);
  threads = clamp_threads(threads, m);
  pthread_t tid[512];
  job_t jobs[512];
  for (int w = 0; w < threads; ++w) {
    job_t j = {t, a, lda, b, ldb, m, n, k, scale, c, ldc, m * w / threads, m * (w + 1) / threads, bdec, NULL,
               sfa, ldsfa, vec, sf_ue4m3};
    jobs[w] = j;
    pthread_create(&tid[w], NULL, f64_rows, &jobs[w]);
  }
  for (int w = 0; w < threads; ++w) pthread_join(tid[w], NULL);
  free(bdec);
  return 0;
}

int kl_oracle_gemm_mx_f64(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                          int64_t k, const uint8_t* sfa, int64_t ldsfa, const uint8_t* sfb, int64_t ldsfb,
                          double scale, double* c, int64_t ldc, int threads) {
  return kl_oracle_gemm_bs_f64(t, a, lda, b, ldb, m, n, k, sfa, ldsfa, sfb, ldsfb, 32, 0, scale, c, ldc, threads);
}

int kl_oracle_gemm_f64(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                       int64_t k, double scale, double* c, int64_t ldc, int threads) {
  return kl_oracle_gemm_mx_f64(t, a, lda, b, ldb, m, n, k, NULL, 0, NULL, 0, scale, c, ldc, threads);
}

/* fp32-accumulate baseline. Blocks of 4 rows of A against 4 rows of B, K in chunks that stay in
 * L1/L2, 8 independent fp32 partial sums per dot so the compiler can vectorise. */
#define KB 512
static void* f32_rows(void* arg) {
  job_t* j = (job_t*)arg;
  const int64_t k = j->k;
  float* c = (float*)j->c;
  float* ablk = (float*)malloc(sizeof(float) * 4 * (size_t)k);
  double* tmp = (double*)malloc(sizeof(double) * (size_t)k);
  for (int64_t i0 = j->row_begin; i0 < j->row_end; i0 += 4) {
    const int64_t ni = (j->row_end - i0) < 4 ? (j->row_end - i0) : 4;
    for (int64_t r = 0; r < ni; ++r) {
      decode_row(j->t, j->a, j->lda, i0 + r, k, j->sfa, j->ldsfa, j->vec, j->sf_ue4m3, tmp);
      for (int64_t kk = 0; kk < k; ++kk) ablk[r * k + kk] = (float)tmp[kk];
    }
    for (int64_t r = ni; r < 4; ++r) memset(ablk + r * k, 0, sizeof(float) * (size_t)k);
    for (int64_t col = 0; col < j->n; ++col) {
      const float* brow = j->bdecf + (size_t)col * (size_t)k;
      float acc[4][8];
      memset(acc, 0, sizeof acc);
      int64_t kk = 0;
      for (; kk + 8 <= k; kk += 8)
        for (int r = 0; r < 4; ++r)
          for (int v = 0; v < 8; ++v) acc[r][v] += ablk[r * k + kk + v] * brow[kk + v];
      for (int r = 0; r < ni; ++r) {
        float s = 0.f;
        for (int v = 0; v < 8; ++v) s += acc[r][v];
        for (int64_t q = kk; q < k; ++q) s += ablk[r * k + q] * brow[q];
        c[(size_t)((i0 + r) * j->ldc + col)] = s * (float)j->scale;
      }
    }
  }
  free(ablk);
  free(tmp);
  return NULL;
}

int kl_oracle_gemm_bs_f32(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                          int64_t k, const uint8_t* sfa, int64_t ldsfa, const uint8_t* sfb, int64_t ldsfb, int vec,
                          int sf_ue4m3, double scale, float* c, int64_t ldc, int threads) {
  if (vec <= 0) return 2;
  float* bdec = (float*)malloc(sizeof(float) * (size_t)n * (size_t)(k > 0 ? k : 1));
  double* tmp = (double*)malloc(sizeof(double) * (size_t)(k > 0 ? k : 1));
  if (!bdec || !tmp) return 1;
  for (int64_t r = 0; r < n; ++r) {
    decode_row(t, b, ldb, r, k, sfb, ldsfb, vec, sf_ue4m3, tmp);
    for (int64_t kk = 0; kk < k; ++kk) bdec[r * k + kk] = (float)tmp[kk];
  }
  free(tmp);
  threads = clamp_threads(threads, m);
  pthread_t tid[512];
  job_t jobs[512];
  for (int w = 0; w < threads; ++w) {
    /* Split rows in multiples of 4 so blocks never straddle workers. */
    int64_t b0 = ((m + 3) / 4) * w / threads * 4, b1 = ((m + 3) / 4) * (w + 1) / threads * 4;
    if (b1 > m) b1 = m;
    if (b0 > m) b0 = m;
    job_t j = {t, a, lda, b, ldb, m, n, k, scale, c, ldc, b0, b1, NULL, bdec, sfa, ldsfa, vec, sf_ue4m3};
    jobs[w] = j;
    pthread_create(&tid[w], NULL, f32_rows, &jobs[w]);
  }
  for (int w = 0; w < threads; ++w) pthread_join(tid[w], NULL);
  free(bdec);
  return 0;
}

int kl_oracle_gemm_mx_f32(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                          int64_t k, const uint8_t* sfa, int64_t ldsfa, const uint8_t* sfb, int64_t ldsfb,
                          double scale, float* c, int64_t ldc, int threads) {
  return kl_oracle_gemm_bs_f32(t, a, lda, b, ldb, m, n, k, sfa, ldsfa, sfb, ldsfb, 32, 0, scale, c, ldc, threads);
}

int kl_oracle_gemm_f32(int t, const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                       int64_t k, double scale, float* c, int64_t ldc, int threads) {
  return kl_oracle_gemm_mx_f32(t, a, lda, b, ldb, m, n, k, NULL, 0, NULL, 0, scale, c, ldc, threads);
}
