/*
 * bm_gemm.h - C ABI of the B200 (sm_100a) FP16 GEMM.
 *
 *   C(M,N) = A(M,K) * B(N,K)^T     FP16 in, FP32 accumulate, FP16 out,
 *                                   alpha = 1, beta = 0, C column-major.
 *
 * This is the drop-in boundary for the hot path of best-matmul. The reference
 * binds its kernels at compile time through the `gemm_backend` namespace
 * (reference: kernels/detail/tma_wgmma_adapter.cuh:134-168, README.md:278-287,
 * benchmark_host.cu:5-10); `kernels/sm100_fp16_gemm.cuh` in this repository
 * keeps that C++ surface as a thin shim over the functions below.
 *
 * Conventions
 *  - All pointers passed as A/B/C are device pointers owned by the caller.
 *    A handle owns only its tensor maps and a 4-byte device status word.
 *  - Functions return BM_OK (0) or a BM_ERR_* code; nothing calls exit().
 *    (The reference calls std::exit on failure, tma_wgmma_adapter.cuh:122-125.)
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - bm_gemm_launch() only enqueues work: it never allocates or synchronises.
 *  - One handle per stream/thread. bm_gemm_prepare() is thread-safe across
 *    handles; launches on different devices from different threads are allowed.
 */
#ifndef BM_GEMM_H_
#define BM_GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BM_GEMM_INTERFACE_VERSION 1 /* reference: benchmark_host.cu:10 (kInterfaceVersion == 1) */

enum bm_status_code {
  BM_OK = 0,
  BM_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size, bad layout characters */
  BM_ERR_UNSUPPORTED_LAYOUT = 2, /* only NT and TN exist (reference host/driver.cuh:101-105) */
  BM_ERR_ALIGNMENT = 3,          /* pointer not 16-byte aligned or leading dimension not x8 */
  BM_ERR_SIZE_LIMIT = 4,         /* element count above INT_MAX (host/driver.cuh:106-113) */
  BM_ERR_CUDA = 5,               /* a CUDA runtime / driver call failed */
  BM_ERR_DEVICE = 6,             /* current device is not compute capability 10.0 */
  BM_ERR_DEVICE_TIMEOUT = 7,     /* a bounded wait inside the kernel expired */
  BM_ERR_VARIANT = 8,            /* unknown variant id, or variant cannot run this shape */
  BM_ERR_TILE_DIVISIBILITY = 9,  /* strict mode: M/N/K not multiples of the tile */
  BM_ERR_SCRATCH_LIMIT = 10      /* bm_gemm_run_noalloc: call needs more scratch than its
                                    static device array holds */
};

/* Kernel variants. BM_VARIANT_AUTO picks one from the shape. */
enum bm_variant {
  BM_VARIANT_AUTO = 0,
  BM_VARIANT_2CTA_256x256 = 1, /* cta_group::2 pair, 256x256 tile, 6 stages */
  BM_VARIANT_1CTA_128x256 = 2, /* cta_group::1, 128x256 tile, 4 stages */
  BM_VARIANT_1CTA_128x128 = 3, /* cta_group::1, 128x128 tile, 6 stages */
  BM_VARIANT_2CTA_256x128 = 4, /* cta_group::2 pair, 256x128 tile, 6 stages */
  BM_VARIANT_2CTA_256x512 = 5  /* cta_group::2 pair, 256x512 tile (two N=256 MMAs share
                                  each A tile; all 512 TMEM columns), 4 stages */
};

/* Problem description. Mirrors gemm_bench::GemmProblem (reference
 * host/common.cuh:47-76): logical A(M,K), B(N,K), C(M,N);
 *   NT ('N','T'): a[m + k*lda], b[n + k*ldb]
 *   TN ('T','N'): a[m*lda + k], b[n*ldb + k]
 *   C           : c[m + n*ldc]
 * lda/ldb/ldc = 0 selects the reference defaults (GemmProblem::ldA/ldB/ldC). */
typedef struct bm_gemm_desc {
  int m, n, k;
  char trans_a, trans_b;
  const void* a;
  const void* b;
  void* c;
  int64_t lda, ldb, ldc;
  int variant;     /* enum bm_variant */
  int strict_tiles; /* non-zero: reject shapes that are not tile multiples, like the
                       reference's validate_problem (tma_wgmma_adapter.cuh:134-141) */
} bm_gemm_desc;

/* Launch geometry reported back to the harness; mirrors
 * gemm_bench::LaunchConfig (reference host/common.cuh:92-97). */
typedef struct bm_launch_info {
  int smem_bytes;
  int grid[3];
  int block[3];
  int cluster[3];
  int variant;
  int tile_m, tile_n, tile_k;
  int stages;
  int num_tiles;
  int cta_group;
} bm_launch_info;

typedef struct bm_gemm_handle bm_gemm_handle;

/* Interface version (== BM_GEMM_INTERFACE_VERSION). */
int bm_gemm_interface_version(void);

/* Human-readable text for a status code (static storage). */
const char* bm_gemm_error_string(int code);

/* Name of a variant, e.g. "sm100_tcgen05_2cta_256x256x64_s6" (static storage);
 * reference: gemm_backend::kName. */
const char* bm_gemm_variant_name(int variant);

/* Validate a problem without touching the GPU (reference:
 * host/driver.cuh:93-114 validate_options + tma_wgmma_adapter.cuh:134-141
 * validate_problem). Returns BM_OK or the first violated rule. */
int bm_gemm_check(const bm_gemm_desc* desc);

/* Build tensor maps and launch geometry once (reference:
 * tma_wgmma_adapter.cuh:57-113, the part of with_prepared_impl before
 * `launch`). Uses the current CUDA device. */
int bm_gemm_prepare(const bm_gemm_desc* desc, bm_gemm_handle** out);

/* Enqueue one GEMM on `stream` (reference: the `launch()` closure,
 * tma_wgmma_adapter.cuh:118-126). No allocation, no synchronisation. */
int bm_gemm_launch(bm_gemm_handle* handle, void* stream);

/* Launch geometry of a prepared handle. */
int bm_gemm_query(const bm_gemm_handle* handle, bm_launch_info* info);

/* Synchronise the device and read (and clear) the kernel status word.
 * Returns BM_OK, BM_ERR_DEVICE_TIMEOUT (bits in *device_bits), or BM_ERR_CUDA. */
int bm_gemm_status(bm_gemm_handle* handle, uint32_t* device_bits);

/* Test hooks: bound on every in-kernel wait (default 2 s) and debug flags
 * (bit 0: the epilogue first waits on a barrier that nothing signals, so the
 * wait must expire and be reported). */
int bm_gemm_set_debug(bm_gemm_handle* handle, uint64_t timeout_ns, uint32_t debug_flags);

void bm_gemm_destroy(bm_gemm_handle* handle);

/* Schedule of the persistent grid. No counterpart in the reference, whose
 * grid is one CTA per output tile (kernels/detail/tma_wgmma_adapter.cuh:96-113)
 * and so leaves its last wave partly idle whenever the tile count is not a
 * multiple of the CTAs resident at once.
 *   BM_SPLIT_AUTO (default) whole tiles fill complete waves; when the tiles
 *                 left for the last wave are at most half the resident
 *                 clusters, they are cut into 256-column halves (full K
 *                 range, one N = 256 MMA per K step) that twice as many
 *                 clusters share. Only the 2-CTA 256x512 variant splits.
 *   BM_SPLIT_NONE whole tiles only.
 * Each output element is still computed by one MMA chain over all of K in the
 * same order, so both modes give the same bits; nothing is allocated and no
 * CTA waits on another. */
enum bm_split_mode { BM_SPLIT_NONE = 0, BM_SPLIT_AUTO = 1 };

typedef struct bm_schedule_info {
  int whole_tiles;       /* tiles computed whole, in full waves */
  int split_tiles;       /* tiles computed in column parts */
  int split_parts;       /* parts of those tiles */
  int split_clusters;    /* clusters sharing the parts */
  int grid_clusters;     /* clusters launched */
  int resident_clusters; /* clusters that fit on the device at once */
  int split_cols;        /* columns per part (0: variant never splits) */
} bm_schedule_info;

/* Re-plan a prepared handle's schedule (mode: enum bm_split_mode). Host-side
 * only: takes effect from the next bm_gemm_launch. */
int bm_gemm_set_split(bm_gemm_handle* handle, int mode);

/* Schedule of a prepared handle. */
int bm_gemm_query_schedule(const bm_gemm_handle* handle, bm_schedule_info* info);

/* Size of the device scratch array used by bm_gemm_run_noalloc (bytes). */
#define BM_NOALLOC_SCRATCH_BYTES 256

/* One GEMM that allocates no device memory. No counterpart in the reference:
 * the reference always allocates (thrust::device_vector buffers and CUTLASS
 * launch state, host/common.cuh:125-145).
 *
 * For callers that cannot call cudaMalloc: programs whose device memory is
 * owned by another allocator (for example a framework's caching allocator
 * that has already reserved the free memory), runtimes that forbid device
 * allocation after start-up, and latency-critical paths where cudaMalloc /
 * cudaFree's implicit device-wide synchronisation is not acceptable.
 *
 * The kernel's only scratch (its 4-byte error word) lives in a file-scope
 * static __device__ array of BM_NOALLOC_SCRATCH_BYTES bytes that every GPU
 * loading the library keeps until the process exits. A call that would need
 * more scratch than that is rejected with BM_ERR_SCRATCH_LIMIT.
 * Set-up: the first call on each device (with that device current) looks up
 * the array's device address and sets the kernel attributes; make that first
 * call before any stream capture. Every call shares the array and clears the
 * error word at its start on `stream`; calls that overlap on the GPU (other
 * streams, other threads) race on it. The caller passes A, B and C as usual.
 * device_status: NULL -> fully asynchronous; non-NULL -> the call waits for
 * `stream` and stores the kernel's error bits there (0 = clean). */
int bm_gemm_run_noalloc(const bm_gemm_desc* desc, void* stream, uint32_t* device_status);

/* Device-side input generator, bit-identical to the CPU oracle's
 * (oracle/bm_oracle.c, bmo_input_value):
 *   mode 0 zero, 1 one, 3 periodic -2..2 on the physical index (reference
 *   host/common.cuh:111-122), 4 uniform[-1,1), 5 normal(0, 0.02) (counter-based
 *   splitmix64 of (seed, matrix_id, logical index) so shards generate their
 *   own rows). Mode 2 (std::rand sequence) is host-only.
 * Writes a logical rows x cols matrix starting at logical row `row0` of a
 * matrix with `total_rows` rows and `cols` columns:
 *   row_major = 1 (K contiguous): dst[r*ld + c]; row_major = 0: dst[r + c*ld].
 * The physical index used by mode 3 is that of the full (total_rows x cols)
 * matrix with leading dimension `full_ld`. */
int bm_fill_fp16(void* dst, int64_t rows, int64_t cols, int64_t ld, int row_major,
                 int64_t row0, int64_t full_ld, int mode, uint64_t seed, int matrix_id,
                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BM_GEMM_H_ */
