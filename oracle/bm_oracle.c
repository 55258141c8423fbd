/*
 * bm_oracle.c - CPU oracle (TEST INFRASTRUCTURE ONLY; see bm_oracle.h).
 *
 * A plain-C restatement of the reference's CPU-side algorithms for the FP16
 * GEMM hot path: input generation (host/common.cuh), the FP64 reference dot
 * product and the sampled validation (host/validation.cuh), and the exact
 * integer full-output check (tests/full_output_validation.cu). Pinned against
 * the reference's own header compiled in place (oracle/ref_shim.cu) by
 * tests/test_oracle.py.
 */
#include "bm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- FP16 */

uint16_t bmo_half_from_float(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof(x));
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFFu) {
    if (man) return (uint16_t)(sign | 0x7E00u | (man >> 13)); /* quiet NaN */
    return (uint16_t)(sign | 0x7C00u);                         /* infinity */
  }
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u); /* overflow -> infinity */
  if (e <= 0) {
    /* binary16 subnormal (or zero): drop 14 - e bits of the 24-bit significand */
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    uint32_t hm = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) ++hm; /* may carry into exponent 1 */
    return (uint16_t)(sign | hm);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may reach infinity */
  return (uint16_t)h;
}

float bmo_float_from_half(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  uint32_t x;
  if (exp == 0) {
    float v = (float)man * 5.9604644775390625e-08f; /* man * 2^-24, exact */
    memcpy(&x, &v, sizeof(x));
    x |= sign;
  } else if (exp == 31) {
    x = sign | 0x7F800000u | (man << 13);
  } else {
    x = sign | ((exp - 15u + 127u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, sizeof(f));
  return f;
}

/* ------------------------------------------------------ index functions */

int64_t bmo_a_index(int nt, int64_t lda, int row, int p) {
  /* host/common.cuh:65-68: NT -> row + p*ldA, TN -> row*ldA + p */
  return nt ? (int64_t)row + (int64_t)p * lda : (int64_t)row * lda + p;
}

int64_t bmo_b_index(int nt, int64_t ldb, int col, int p) {
  /* host/common.cuh:69-72: NT (transB == 'T') -> col + p*ldB, TN -> col*ldB + p */
  return nt ? (int64_t)col + (int64_t)p * ldb : (int64_t)col * ldb + p;
}

/* ------------------------------------------------------ input generation */

static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t gen_key(uint64_t seed, int matrix_id) {
  return mix64(seed ^ ((uint64_t)matrix_id * 0xD1B54A32D192ED03ull));
}

static uint64_t gen_bits(uint64_t key, uint64_t index) {
  return mix64(key + (index + 1ull) * 0x9E3779B97F4A7C15ull);
}

static float gen_value_f32(int mode, uint64_t key, uint64_t logical, uint64_t physical,
                           int matrix_id) {
  switch (mode) {
    case 0: return 0.0f;
    case 1: return 1.0f;
    case 3: /* host/common.cuh:117-119 */
      return (float)((int)((physical + (uint64_t)matrix_id * 17ull) % 5ull) - 2);
    case 4: {
      const uint32_t u = (uint32_t)(gen_bits(key, logical) >> 40);
      return (float)u * (1.0f / 8388608.0f) - 1.0f;
    }
    case 5: {
      const uint64_t b0 = gen_bits(key, 2ull * logical);
      const uint64_t b1 = gen_bits(key, 2ull * logical + 1ull);
      int32_t s = 0;
      for (int i = 0; i < 4; ++i) {
        s += (int32_t)((b0 >> (16 * i)) & 0xFFFFu);
        s += (int32_t)((b1 >> (16 * i)) & 0xFFFFu);
      }
      return (float)(s - 262140) * 3.7376248e-07f;
    }
    default: return 0.0f;
  }
}

uint16_t bmo_input_value(int mode, uint64_t seed, int matrix_id, uint64_t logical_index,
                         uint64_t physical_index) {
  return bmo_half_from_float(
      gen_value_f32(mode, gen_key(seed, matrix_id), logical_index, physical_index, matrix_id));
}

void bmo_make_inputs(int m, int n, int k, int nt, int mode, uint64_t seed, uint16_t* a,
                     uint16_t* b) {
  const int64_t na = (int64_t)m * k, nb = (int64_t)n * k;
  if (mode == 2) {
    /* host/common.cuh:134-140 with make_input_value mode RandomPm1 (:116):
     * one std::rand() per element, A first, then B, in physical order. */
    const uint16_t one = bmo_half_from_float(1.0f), neg = bmo_half_from_float(-1.0f);
    srand(0);
    for (int64_t i = 0; i < na; ++i) a[i] = (rand() % 2) ? one : neg;
    for (int64_t i = 0; i < nb; ++i) b[i] = (rand() % 2) ? one : neg;
    return;
  }
  const uint64_t ka = gen_key(seed, 0), kb = gen_key(seed, 1);
  for (int64_t i = 0; i < na; ++i) {
    /* logical (row, p) of physical index i */
    const int64_t row = nt ? i % m : i / k, p = nt ? i / m : i % k;
    a[i] = bmo_half_from_float(gen_value_f32(mode, ka, (uint64_t)(row * k + p), (uint64_t)i, 0));
  }
  for (int64_t i = 0; i < nb; ++i) {
    const int64_t col = nt ? i % n : i / k, p = nt ? i / n : i % k;
    b[i] = bmo_half_from_float(gen_value_f32(mode, kb, (uint64_t)(col * k + p), (uint64_t)i, 1));
  }
}

void bmo_fill(uint16_t* dst, int64_t rows, int64_t cols, int64_t ld, int row_major, int64_t row0,
              int64_t full_ld, int mode, uint64_t seed, int matrix_id) {
  const uint64_t key = gen_key(seed, matrix_id);
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t gr = row0 + r;
      const uint64_t logical = (uint64_t)gr * (uint64_t)cols + (uint64_t)c;
      const uint64_t physical = row_major ? (uint64_t)(gr * full_ld + c) : (uint64_t)(gr + c * full_ld);
      const int64_t off = row_major ? r * ld + c : r + c * ld;
      dst[off] = bmo_half_from_float(gen_value_f32(mode, key, logical, physical, matrix_id));
    }
  }
}

/* ------------------------------------------------------ reference GEMM */

double bmo_gemm_entry_f64(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b,
                          int64_t ldb, int row, int col) {
  /* host/validation.cuh:31-42: FP64 sum over p of double(float(A)) * double(float(B)) */
  double acc = 0.0;
  for (int p = 0; p < k; ++p) {
    acc += (double)bmo_float_from_half(a[bmo_a_index(nt, lda, row, p)]) *
           (double)bmo_float_from_half(b[bmo_b_index(nt, ldb, col, p)]);
  }
  return acc;
}

typedef struct {
  int k, nt;
  const uint16_t *a, *b;
  int64_t lda, ldb;
  const int *rows, *cols;
  int64_t begin, end;
  double* out;
} EntriesJob;

static void* entries_worker(void* arg) {
  EntriesJob* j = (EntriesJob*)arg;
  for (int64_t i = j->begin; i < j->end; ++i)
    j->out[i] = bmo_gemm_entry_f64(j->k, j->nt, j->a, j->lda, j->b, j->ldb, j->rows[i], j->cols[i]);
  return NULL;
}

void bmo_gemm_entries_f64(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b,
                          int64_t ldb, const int* rows, const int* cols, int64_t count,
                          double* out, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  EntriesJob job[256];
  for (int t = 0; t < threads; ++t) {
    job[t] = (EntriesJob){k, nt, a, b, lda, ldb, rows, cols, count * t / threads,
                          count * (t + 1) / threads, out};
    pthread_create(&tid[t], NULL, entries_worker, &job[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
}

typedef struct {
  int k, nt;
  const uint16_t *a, *b;
  int64_t lda, ldb;
  int row0, rows, col0, cols;
  int c_begin, c_end;
  const float* af; /* A block as float, row-major [rows][k] */
  float* out;
} F32Job;

static void* f32_worker(void* arg) {
  F32Job* j = (F32Job*)arg;
  float* bcol = (float*)malloc(sizeof(float) * (size_t)j->k);
  for (int c = j->c_begin; c < j->c_end; ++c) {
    const int col = j->col0 + c;
    for (int p = 0; p < j->k; ++p) bcol[p] = bmo_float_from_half(j->b[bmo_b_index(j->nt, j->ldb, col, p)]);
    for (int r = 0; r < j->rows; ++r) {
      const float* ar = j->af + (size_t)r * j->k;
      float acc = 0.0f;
      for (int p = 0; p < j->k; ++p) acc += ar[p] * bcol[p];
      j->out[(int64_t)r + (int64_t)c * j->rows] = acc;
    }
  }
  free(bcol);
  return NULL;
}

void bmo_gemm_f32(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb,
                  int row0, int rows, int col0, int cols, float* out, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  float* af = (float*)malloc(sizeof(float) * (size_t)rows * (size_t)k);
  for (int r = 0; r < rows; ++r)
    for (int p = 0; p < k; ++p)
      af[(size_t)r * k + p] = bmo_float_from_half(a[bmo_a_index(nt, lda, row0 + r, p)]);
  pthread_t tid[256];
  F32Job job[256];
  for (int t = 0; t < threads; ++t) {
    job[t] = (F32Job){k, nt, a, b, lda, ldb, row0, rows, col0, cols,
                      (int)((int64_t)cols * t / threads), (int)((int64_t)cols * (t + 1) / threads),
                      af, out};
    pthread_create(&tid[t], NULL, f32_worker, &job[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(af);
}

int bmo_gemm_exact_int(int m, int n, int k, int nt, const uint16_t* a, const uint16_t* b,
                       int32_t* out) {
  /* tests/full_output_validation.cu:84-101: integer dot products; every
   * partial sum must stay within +-2048 (exact in FP16). */
  const int64_t lda = nt ? m : k, ldb = nt ? n : k;
  for (int col = 0; col < n; ++col) {
    for (int row = 0; row < m; ++row) {
      int expected = 0;
      for (int p = 0; p < k; ++p) {
        expected += (int)bmo_float_from_half(a[bmo_a_index(nt, lda, row, p)]) *
                    (int)bmo_float_from_half(b[bmo_b_index(nt, ldb, col, p)]);
        if (abs(expected) > 2048) return -1;
      }
      out[(int64_t)row + (int64_t)col * m] = expected;
    }
  }
  return 0;
}

int64_t bmo_check(const uint16_t* c, const double* ref, int64_t count, int k, double rtol,
                  double atol, double* max_err, int64_t* worst) {
  const double abs_term = atol * sqrt((double)k / 4096.0);
  int64_t bad = 0, worst_i = -1;
  double merr = 0.0, wratio = -1.0;
  for (int64_t i = 0; i < count; ++i) {
    const double v = (double)bmo_float_from_half(c[i]);
    const double err = fabs(v - ref[i]);
    const double tol = rtol * fabs(ref[i]) + abs_term;
    if (!(err <= tol)) ++bad; /* NaN counts as a violation */
    if (err > merr || err != err) merr = err;
    const double ratio = err / tol;
    if (!(ratio <= wratio)) {
      wratio = ratio;
      worst_i = i;
    }
  }
  if (max_err) *max_err = merr;
  if (worst) *worst = worst_i;
  return bad;
}

int bmo_validate_sampled(int m, int n, int k, int nt, const uint16_t* a, int64_t lda,
                         const uint16_t* b, int64_t ldb, const uint16_t* c, int64_t ldc,
                         double* max_abs_error, double* checksum) {
  /* host/validation.cuh:12-27 (finite scan + checksum) and :47-75 (4x4 grid,
   * tolerance 1 + 0.02*|reference|, host/common.cuh:106-108). */
  double sum = 0.0;
  for (int col = 0; col < n; ++col)
    for (int row = 0; row < m; ++row) {
      const double v = (double)bmo_float_from_half(c[(int64_t)row + (int64_t)col * ldc]);
      if (!isfinite(v)) return 1 + 16;
      sum += v;
    }
  double merr = 0.0;
  for (int r = 0; r < 4; ++r) {
    const int row = (int)((long long)(m - 1) * r / 3);
    for (int cc = 0; cc < 4; ++cc) {
      const int col = (int)((long long)(n - 1) * cc / 3);
      const double ref = bmo_gemm_entry_f64(k, nt, a, lda, b, ldb, row, col);
      const double actual = (double)bmo_float_from_half(c[(int64_t)row + (int64_t)col * ldc]);
      const double err = fabs(actual - ref);
      if (err > merr) merr = err;
      if (err > 1.0 + 0.02 * fabs(ref)) {
        if (max_abs_error) *max_abs_error = merr;
        if (checksum) *checksum = sum;
        return 1 + r * 4 + cc;
      }
    }
  }
  if (max_abs_error) *max_abs_error = merr;
  if (checksum) *checksum = sum;
  return 0;
}
