/*
 * bm_oracle.h - CPU oracle for the FP16 GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: the tests, the
 * smoke check and bench.py's CPU-baseline leg call it to judge the CUDA path.
 * Nothing in the product (best-matmul_b200/) links or calls it.
 *
 * Every function restates an algorithm of the reference (ggbond-x/best-matmul)
 * in plain C; the reference file:line it follows is cited at each function.
 * FP16 values are passed as raw IEEE binary16 bit patterns (uint16_t).
 */
#ifndef BM_ORACLE_H_
#define BM_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32, round-to-nearest-even (cutlass::half_t semantics
 * used by the reference's Element type, host/common.cuh:19). */
uint16_t bmo_half_from_float(float f);
float bmo_float_from_half(uint16_t h);

/* Physical index functions of gemm_bench::GemmProblem (host/common.cuh:54-75). */
int64_t bmo_a_index(int nt, int64_t lda, int row, int p);
int64_t bmo_b_index(int nt, int64_t ldb, int col, int p);

/* Input generation.
 * Modes 0..3 restate GemmBuffers (host/common.cuh:125-144) with
 * make_input_value (host/common.cuh:111-122): srand(0), then A in physical
 * order (matrix_id 0), then B (matrix_id 1). Mode 2 draws std::rand() % 2.
 * Modes 4/5 are the counter-based generators of the device fill kernel
 * (best-matmul_b200/csrc/bm_inputs.cuh), restated here bit for bit. */
void bmo_make_inputs(int m, int n, int k, int nt, int mode, uint64_t seed,
                     uint16_t* a, uint16_t* b);

/* One value of the counter-based generators (modes 0, 1, 3, 4, 5). */
uint16_t bmo_input_value(int mode, uint64_t seed, int matrix_id, uint64_t logical_index,
                         uint64_t physical_index);

/* Fill a logical rows x cols block starting at logical row row0, as
 * bm_fill_fp16 does on the device (same argument meaning). */
void bmo_fill(uint16_t* dst, int64_t rows, int64_t cols, int64_t ld, int row_major, int64_t row0,
              int64_t full_ld, int mode, uint64_t seed, int matrix_id);

/* reference_gemm_entry (host/validation.cuh:31-42): one C(row, col) with
 * FP64 accumulation of FP16 products. */
double bmo_gemm_entry_f64(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b,
                          int64_t ldb, int row, int col);

/* FP64 entries for a list of (row, col) samples, on `threads` threads. */
void bmo_gemm_entries_f64(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b,
                          int64_t ldb, const int* rows, const int* cols, int64_t count,
                          double* out, int threads);

/* FP32-accumulate twin of the same dot product for every C(row, col) with
 * row in [row0, row0+rows), col in [col0, col0+cols): out[r + c*rows]
 * (column-major, like C). Products are summed in k order. */
void bmo_gemm_f32(int k, int nt, const uint16_t* a, int64_t lda, const uint16_t* b, int64_t ldb,
                  int row0, int rows, int col0, int cols, float* out, int threads);

/* Integer reference for the exact-output regressions of
 * tests/full_output_validation.cu:84-101: returns 0 and fills out[] (int32,
 * column-major rows x cols) when every partial sum stays within +-2048,
 * else -1. */
int bmo_gemm_exact_int(int m, int n, int k, int nt, const uint16_t* a, const uint16_t* b,
                       int32_t* out);

/* Tolerance check |c - ref| <= rtol*|ref| + atol*sqrt(K/4096) on every entry.
 * c: FP16 bits, ref: double, both length count. Returns the number of
 * violations; *max_err and *worst (index of the worst ratio) are reported. */
int64_t bmo_check(const uint16_t* c, const double* ref, int64_t count, int k, double rtol,
                  double atol, double* max_err, int64_t* worst);

/* Sampled grid check of validate_gemm_output (host/validation.cuh:47-75):
 * 4 x 4 evenly spaced (row, col) including the corners, tolerance
 * 1 + 0.02*|ref|. Returns 0 on pass, else 1 + index of the failing sample. */
int bmo_validate_sampled(int m, int n, int k, int nt, const uint16_t* a, int64_t lda,
                         const uint16_t* b, int64_t ldb, const uint16_t* c, int64_t ldc,
                         double* max_abs_error, double* checksum);

#ifdef __cplusplus
}
#endif

#endif /* BM_ORACLE_H_ */
