// C ABI of the sm_100a FP16 GEMM (declared in include/bm_gemm.h).
//
// bm_gemm_prepare() does, once, what the reference's with_prepared_impl does
// before handing out `launch` (kernels/detail/tma_wgmma_adapter.cuh:57-113):
// validate the problem, encode TMA descriptors, pick the launch geometry and
// raise the dynamic shared-memory limit. bm_gemm_launch() is the `launch()`
// closure (tma_wgmma_adapter.cuh:118-126): one cudaLaunchKernelEx on the
// caller's stream, no allocation, no synchronisation.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "../../include/bm_gemm.h"
#include "bm_inputs.cuh"
#include "gemm_sm100.cuh"
#include "schedule.cuh"

namespace {

using bm::GemmConfig;
using bm::GemmParams;

constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s bound on every in-kernel wait

struct VariantInfo {
  int id;
  const char* name;
  int cta_group;
  int mma_n;   // N of one MMA instruction
  int num_n;   // MMAs per K step sharing one A tile
  int stages;
};

// X(id, cta_group, mma_n, num_n, stages): every compiled kernel variant.
#define BM_FOR_EACH_VARIANT(X)                 \
  X(BM_VARIANT_2CTA_256x256, 2, 256, 1, 6)     \
  X(BM_VARIANT_1CTA_128x256, 1, 256, 1, 4)     \
  X(BM_VARIANT_1CTA_128x128, 1, 128, 1, 6)     \
  X(BM_VARIANT_2CTA_256x128, 2, 128, 1, 6)     \
  X(BM_VARIANT_2CTA_256x512, 2, 256, 2, 4)

const VariantInfo kVariants[] = {
    {BM_VARIANT_AUTO, "auto", 0, 0, 0, 0},
    {BM_VARIANT_2CTA_256x256, "sm100_tcgen05_2cta_256x256x64_s6", 2, 256, 1, 6},
    {BM_VARIANT_1CTA_128x256, "sm100_tcgen05_1cta_128x256x64_s4", 1, 256, 1, 4},
    {BM_VARIANT_1CTA_128x128, "sm100_tcgen05_1cta_128x128x64_s6", 1, 128, 1, 6},
    {BM_VARIANT_2CTA_256x128, "sm100_tcgen05_2cta_256x128x64_s6", 2, 128, 1, 6},
    {BM_VARIANT_2CTA_256x512, "sm100_tcgen05_2cta_256x512x64_s4", 2, 256, 2, 4},
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);

using LaunchFn = cudaError_t (*)(const bm_gemm_handle*, cudaStream_t);

}  // namespace

struct bm_gemm_handle {
  CUtensorMap tmap_a;
  CUtensorMap tmap_b;
  CUtensorMap tmap_c;
  GemmParams params;
  int variant;
  bool nt;
  int cta_group;
  int tile_m, tile_n, stages;
  int grid;
  int smem_bytes;
  int device;
  uint32_t* d_status;
  LaunchFn launch;
  int max_clusters;  // resident clusters of this variant on this device
  int parts;         // column parts per tile the variant can split into (1: none)
  int split_mode;    // enum bm_split_mode
};

namespace {

template <int kCtaGroup, int kBN, int kNumN, int kStages, bool kMn>
cudaError_t launch_variant(const bm_gemm_handle* h, cudaStream_t stream) {
  using Cfg = GemmConfig<kCtaGroup, kBN, kNumN, kStages, kMn>;
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(h->grid), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(Cfg::kSmemBytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCtaGroup;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: this grid's CTAs may be scheduled while
  // the previous kernel in the stream finishes; the kernel waits for that
  // kernel's completion (griddepcontrol.wait) before touching global memory.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, bm::bm_gemm_sm100_kernel<kCtaGroup, kBN, kNumN, kStages, kMn>,
                            h->tmap_a, h->tmap_b, h->tmap_c, h->params);
}

// Per (device, variant, layout): shared-memory attribute set and resident
// cluster count. Guarded by a mutex; computed on first prepare.
struct GeometryCache {
  bool ready = false;
  int max_clusters = 0;
};
std::mutex g_cache_mutex;
GeometryCache g_cache[64][kNumVariants][2];

template <int kCtaGroup, int kBN, int kNumN, int kStages, bool kMn>
cudaError_t geometry(int device, int sm_count, int variant, int* max_clusters, int* smem) {
  using Cfg = GemmConfig<kCtaGroup, kBN, kNumN, kStages, kMn>;
  static_assert(Cfg::kSmemBytes > 116 * 1024,
                "one CTA per SM is required: each CTA allocates all the TMEM it uses");
  *smem = Cfg::kSmemBytes;
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  GeometryCache& gc = g_cache[device & 63][variant][kMn ? 1 : 0];
  if (gc.ready) {
    *max_clusters = gc.max_clusters;
    return cudaSuccess;
  }
  auto kernel = bm::bm_gemm_sm100_kernel<kCtaGroup, kBN, kNumN, kStages, kMn>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  int clusters = sm_count / kCtaGroup;
  if (kCtaGroup > 1) {
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count), 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(Cfg::kSmemBytes);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCtaGroup;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    if (e != cudaSuccess) return e;
    if (n > 0 && n < clusters) clusters = n;
  }
  gc.ready = true;
  gc.max_clusters = clusters;
  *max_clusters = clusters;
  return cudaSuccess;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// 2D FP16 tensor map: dim0 (contiguous) x dim1 with row pitch ld elements.
bool encode_2d(CUtensorMap* map, const void* ptr, uint64_t dim0, uint64_t dim1, uint64_t ld,
               uint32_t box0, uint32_t box1, bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct Resolved {
  bool nt;
  int64_t lda, ldb, ldc;
};

int resolve(const bm_gemm_desc* d, Resolved* r) {
  if (!d) return BM_ERR_INVALID_ARGUMENT;
  if (d->m <= 0 || d->n <= 0 || d->k <= 0) return BM_ERR_INVALID_ARGUMENT;
  const bool nt = d->trans_a == 'N' && d->trans_b == 'T';
  const bool tn = d->trans_a == 'T' && d->trans_b == 'N';
  if (!nt && !tn) return BM_ERR_UNSUPPORTED_LAYOUT;
  const uint64_t lim = static_cast<uint64_t>(INT_MAX);
  const uint64_t m = d->m, n = d->n, k = d->k;
  if (m * k > lim || n * k > lim || m * n > lim) return BM_ERR_SIZE_LIMIT;
  r->nt = nt;
  r->lda = d->lda ? d->lda : (nt ? d->m : d->k);
  r->ldb = d->ldb ? d->ldb : (nt ? d->n : d->k);
  r->ldc = d->ldc ? d->ldc : d->m;
  const int64_t min_lda = nt ? d->m : d->k;
  const int64_t min_ldb = nt ? d->n : d->k;
  if (r->lda < min_lda || r->ldb < min_ldb || r->ldc < d->m) return BM_ERR_INVALID_ARGUMENT;
  // TMA: row pitches multiples of 16 bytes, base addresses 16-byte aligned.
  if ((r->lda % 8) || (r->ldb % 8) || (r->ldc % 8)) return BM_ERR_ALIGNMENT;
  return BM_OK;
}

// Column parts a variant's leftover tiles can be split into (1 = whole
// tiles only): the 256x512 pair tile (GemmConfig::kTailSplit).
int split_parts(int variant) {
  const VariantInfo& vi = kVariants[variant];
  return (vi.cta_group == 2 && vi.mma_n == 256 && vi.num_n == 2) ? (vi.mma_n * vi.num_n) / bm::kSplitCols
                                                                   : 1;
}

void apply_plan(bm_gemm_handle* h) {
  GemmParams& p = h->params;
  const bm::Plan pl = bm::plan_schedule(p.num_tiles, h->parts, h->max_clusters,
                                        h->split_mode == BM_SPLIT_AUTO ? 1 : 0);
  p.dp_tiles = pl.dp_tiles;
  p.tail_parts = pl.tail_parts;
  p.tail_clusters = pl.tail_clusters;
  h->grid = pl.grid_clusters * h->cta_group;
}

// Automatic variant choice: estimated throughput = (relative per-tile
// efficiency of the variant, measured on B200) x (fraction of the persistent
// grid kept busy, i.e. wave quantization of the tile count over the resident
// clusters). Skinny M (<= 128) streams B from HBM and takes the 1-CTA
// 128x256 tile, which measured fastest there.
int pick_variant(const bm_gemm_desc* d) {
  if (d->variant != BM_VARIANT_AUTO) return d->variant;
  if (d->m <= 128) return (d->n >= 256) ? BM_VARIANT_1CTA_128x256 : BM_VARIANT_1CTA_128x128;
  static const struct { int id; double eff; } cand[] = {
      {BM_VARIANT_2CTA_256x512, 1.00}, {BM_VARIANT_2CTA_256x256, 0.93},
      {BM_VARIANT_1CTA_128x256, 0.88}, {BM_VARIANT_1CTA_128x128, 0.80}};
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int best = BM_VARIANT_2CTA_256x512;
  double best_score = -1.0;
  for (const auto& c : cand) {
    const VariantInfo& vi = kVariants[c.id];
    const long long tm = 128LL * vi.cta_group, tn = static_cast<long long>(vi.mma_n) * vi.num_n;
    const long long tiles = ((d->m + tm - 1) / tm) * ((d->n + tn - 1) / tn);
    const int slots = sms / vi.cta_group;
    // waves as scheduled (leftover tiles split into halves where that pays)
    const bm::Plan pl = bm::plan_schedule(static_cast<int>(tiles), split_parts(c.id), slots, 1);
    const double busy = static_cast<double>(tiles) / (static_cast<double>(slots) * pl.est);
    const double score = c.eff * busy;
    if (score > best_score + 1e-9) {
      best_score = score;
      best = c.id;
    }
  }
  return best;
}

}  // namespace

extern "C" {

int bm_gemm_interface_version(void) { return BM_GEMM_INTERFACE_VERSION; }

const char* bm_gemm_error_string(int code) {
  switch (code) {
    case BM_OK: return "ok";
    case BM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BM_ERR_UNSUPPORTED_LAYOUT: return "only NT and TN layouts are implemented (use N T or T N)";
    case BM_ERR_ALIGNMENT: return "pointers must be 16-byte aligned and leading dimensions multiples of 8";
    case BM_ERR_SIZE_LIMIT: return "matrix element count exceeds supported range (INT_MAX)";
    case BM_ERR_CUDA: return "CUDA runtime or driver error";
    case BM_ERR_DEVICE: return "device is not compute capability 10.0 (B200 / sm_100a)";
    case BM_ERR_DEVICE_TIMEOUT: return "a bounded wait inside the GEMM kernel expired";
    case BM_ERR_VARIANT: return "unknown kernel variant";
    case BM_ERR_TILE_DIVISIBILITY: return "selected kernel requires M % CTA_M == 0, N % CTA_N == 0, K % CTA_K == 0";
    case BM_ERR_SCRATCH_LIMIT: return "call needs more scratch than the no-alloc entry point's static device array holds";
    default: return "unknown error";
  }
}

const char* bm_gemm_variant_name(int variant) {
  for (const auto& v : kVariants)
    if (v.id == variant) return v.name;
  return "unknown";
}

int bm_gemm_check(const bm_gemm_desc* d) {
  Resolved r;
  int rc = resolve(d, &r);
  if (rc != BM_OK) return rc;
  if (!d->a || !d->b || !d->c) return BM_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(d->a) | reinterpret_cast<uintptr_t>(d->b) |
       reinterpret_cast<uintptr_t>(d->c)) & 15u)
    return BM_ERR_ALIGNMENT;
  const int v = pick_variant(d);
  if (v <= 0 || v >= kNumVariants) return BM_ERR_VARIANT;
  if (d->strict_tiles) {
    const int tm = 128 * kVariants[v].cta_group, tn = kVariants[v].mma_n * kVariants[v].num_n;
    if (d->m % tm || d->n % tn || d->k % 64) return BM_ERR_TILE_DIVISIBILITY;
  }
  return BM_OK;
}

int bm_gemm_prepare(const bm_gemm_desc* d, bm_gemm_handle** out) {
  if (!out) return BM_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int rc = bm_gemm_check(d);
  if (rc != BM_OK) return rc;
  Resolved r;
  resolve(d, &r);
  const int v = pick_variant(d);

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return BM_ERR_CUDA;
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return BM_ERR_CUDA;
  if (major != 10 || minor != 0) return BM_ERR_DEVICE;

  bm_gemm_handle* h = new (std::nothrow) bm_gemm_handle();
  if (!h) return BM_ERR_CUDA;
  h->variant = v;
  h->nt = r.nt;
  h->device = device;
  h->cta_group = kVariants[v].cta_group;
  h->tile_m = 128 * h->cta_group;
  h->tile_n = kVariants[v].mma_n * kVariants[v].num_n;
  h->stages = kVariants[v].stages;

  const int rows_b = kVariants[v].mma_n / h->cta_group;  // B rows per CTA per MMA
  bool ok;
  if (r.nt) {
    ok = encode_2d(&h->tmap_a, d->a, d->m, d->k, r.lda, 64, 64, true) &&
         encode_2d(&h->tmap_b, d->b, d->n, d->k, r.ldb, 64, 64, true);
  } else {
    ok = encode_2d(&h->tmap_a, d->a, d->k, d->m, r.lda, 64, 128, true) &&
         encode_2d(&h->tmap_b, d->b, d->k, d->n, r.ldb, 64, static_cast<uint32_t>(rows_b), true);
  }
  ok = ok && encode_2d(&h->tmap_c, d->c, d->m, d->n, r.ldc, 32, 32, false);
  if (!ok) {
    delete h;
    return BM_ERR_CUDA;
  }

  int max_clusters = 0, smem = 0;
  cudaError_t e = cudaErrorInvalidValue;
  switch (v * 2 + (r.nt ? 1 : 0)) {
#define BM_CASE(VID, CG, BN, NN, ST)                                                    \
  case VID * 2 + 0:                                                                     \
    e = geometry<CG, BN, NN, ST, false>(device, sms, VID, &max_clusters, &smem);        \
    h->launch = &launch_variant<CG, BN, NN, ST, false>;                                 \
    break;                                                                              \
  case VID * 2 + 1:                                                                     \
    e = geometry<CG, BN, NN, ST, true>(device, sms, VID, &max_clusters, &smem);         \
    h->launch = &launch_variant<CG, BN, NN, ST, true>;                                  \
    break;
    BM_FOR_EACH_VARIANT(BM_CASE)
#undef BM_CASE
    default: break;
  }
  if (e != cudaSuccess || max_clusters <= 0) {
    delete h;
    return BM_ERR_CUDA;
  }
  h->smem_bytes = smem;

  GemmParams& p = h->params;
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.tiles_m = (d->m + h->tile_m - 1) / h->tile_m;
  p.tiles_n = (d->n + h->tile_n - 1) / h->tile_n;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (d->k + 63) / 64;
  p.group_m = 8;
  p.timeout_ns = kDefaultTimeoutNs;
  p.debug = 0;
  p.stats = nullptr;
  h->max_clusters = max_clusters;
  h->parts = split_parts(v);
  h->split_mode = BM_SPLIT_AUTO;
  apply_plan(h);

  if (cudaMalloc(reinterpret_cast<void**>(&h->d_status), sizeof(uint32_t)) != cudaSuccess) {
    delete h;
    return BM_ERR_CUDA;
  }
  if (cudaMemset(h->d_status, 0, sizeof(uint32_t)) != cudaSuccess) {
    cudaFree(h->d_status);
    delete h;
    return BM_ERR_CUDA;
  }
  p.status = h->d_status;
  *out = h;
  return BM_OK;
}

int bm_gemm_launch(bm_gemm_handle* h, void* stream) {
  if (!h) return BM_ERR_INVALID_ARGUMENT;
  cudaError_t e = h->launch(h, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? BM_OK : BM_ERR_CUDA;
}

int bm_gemm_query(const bm_gemm_handle* h, bm_launch_info* info) {
  if (!h || !info) return BM_ERR_INVALID_ARGUMENT;
  std::memset(info, 0, sizeof(*info));
  info->smem_bytes = h->smem_bytes;
  info->grid[0] = h->grid;
  info->grid[1] = info->grid[2] = 1;
  info->block[0] = bm::kGemmThreads;
  info->block[1] = info->block[2] = 1;
  info->cluster[0] = h->cta_group;
  info->cluster[1] = info->cluster[2] = 1;
  info->variant = h->variant;
  info->tile_m = h->tile_m;
  info->tile_n = h->tile_n;
  info->tile_k = 64;
  info->stages = h->stages;
  info->num_tiles = h->params.num_tiles;
  info->cta_group = h->cta_group;
  return BM_OK;
}

int bm_gemm_status(bm_gemm_handle* h, uint32_t* bits) {
  if (!h) return BM_ERR_INVALID_ARGUMENT;
  if (cudaDeviceSynchronize() != cudaSuccess) return BM_ERR_CUDA;
  uint32_t v = 0;
  if (cudaMemcpy(&v, h->d_status, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess)
    return BM_ERR_CUDA;
  if (cudaMemset(h->d_status, 0, sizeof(uint32_t)) != cudaSuccess) return BM_ERR_CUDA;
  if (bits) *bits = v;
  return v ? BM_ERR_DEVICE_TIMEOUT : BM_OK;
}

int bm_gemm_set_debug(bm_gemm_handle* h, uint64_t timeout_ns, uint32_t flags) {
  if (!h || timeout_ns == 0) return BM_ERR_INVALID_ARGUMENT;
  h->params.timeout_ns = timeout_ns;
  h->params.debug = flags;
  return BM_OK;
}

int bm_gemm_set_split(bm_gemm_handle* h, int mode) {
  if (!h || (mode != BM_SPLIT_NONE && mode != BM_SPLIT_AUTO)) return BM_ERR_INVALID_ARGUMENT;
  h->split_mode = mode;
  apply_plan(h);
  return BM_OK;
}

int bm_gemm_query_schedule(const bm_gemm_handle* h, bm_schedule_info* info) {
  if (!h || !info) return BM_ERR_INVALID_ARGUMENT;
  std::memset(info, 0, sizeof(*info));
  const GemmParams& p = h->params;
  info->whole_tiles = p.dp_tiles;
  info->split_tiles = p.num_tiles - p.dp_tiles;
  info->split_parts = p.tail_parts;
  info->split_clusters = p.tail_clusters;
  info->grid_clusters = h->grid / h->cta_group;
  info->resident_clusters = h->max_clusters;
  info->split_cols = h->parts > 1 ? bm::kSplitCols : 0;
  return BM_OK;
}

#if defined(BM_KERNEL_STATS)
// Diagnostics builds only (not declared in the public header): attach a
// device buffer of grid x 16 uint64 counters to a handle.
int bm_gemm_debug_attach_stats(bm_gemm_handle* h, void* stats) {
  if (!h) return BM_ERR_INVALID_ARGUMENT;
  h->params.stats = static_cast<unsigned long long*>(stats);
  return BM_OK;
}
#endif

void bm_gemm_destroy(bm_gemm_handle* h) {
  if (!h) return;
  if (h->d_status) cudaFree(h->d_status);
  delete h;
}

}  // extern "C"

// ------------------------------------------------------------------ inputs
namespace {

__global__ void fill_fp16_kernel(__half* dst, int64_t rows, int64_t cols, int64_t ld, int row_major,
                                 int64_t row0, int64_t full_ld, int mode, uint64_t key, int mid) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r, c;
    if (row_major) {
      r = i / cols;
      c = i - r * cols;
    } else {
      c = i / rows;
      r = i - c * rows;
    }
    const int64_t gr = row0 + r;
    const uint64_t logical = static_cast<uint64_t>(gr) * static_cast<uint64_t>(cols) + c;
    const uint64_t physical = row_major ? static_cast<uint64_t>(gr * full_ld + c)
                                        : static_cast<uint64_t>(gr + c * full_ld);
    const float v = bm::input_value_f32(mode, key, logical, physical, mid);
    const int64_t off = row_major ? r * ld + c : r + c * ld;
    dst[off] = __float2half_rn(v);
  }
}

}  // namespace

extern "C" int bm_fill_fp16(void* dst, int64_t rows, int64_t cols, int64_t ld, int row_major,
                            int64_t row0, int64_t full_ld, int mode, uint64_t seed, int matrix_id,
                            void* stream) {
  if (!dst || rows <= 0 || cols <= 0 || row0 < 0) return BM_ERR_INVALID_ARGUMENT;
  if (mode < 0 || mode > 5 || mode == 2) return BM_ERR_INVALID_ARGUMENT;
  if (row_major ? (ld < cols) : (ld < rows)) return BM_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return BM_ERR_CUDA;
  const uint64_t key = bm::input_key(seed, matrix_id);
  fill_fp16_kernel<<<sms * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(dst), rows, cols, ld, row_major, row0, full_ld, mode, key, matrix_id);
  return cudaGetLastError() == cudaSuccess ? BM_OK : BM_ERR_CUDA;
}

// ------------------------------------------------------- no-alloc entry point
// bm_gemm_run_noalloc: the same GEMM kernel, launched without any device
// allocation, for callers that cannot call cudaMalloc (memory owned by another
// allocator, no device allocation allowed after start-up, or no tolerance for
// cudaMalloc/cudaFree's device-wide synchronisation).
//
// The kernel's scratch is its error word. Here it lives in a file-scope
// device array instead of a cudaMalloc'd buffer. Host code must not use the
// array's name as a device address: its device address is looked up with
// cudaGetSymbolAddress once per device (with that device current) on the
// first call, and that pointer is what the kernel receives.
namespace {

constexpr size_t kNoAllocScratchBytes = BM_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(uint32_t)];

// Scratch one call needs: the kernel's single 32-bit error word.
constexpr size_t kNoAllocScratchPerCall = sizeof(uint32_t);

struct NoAllocDevice {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  uint32_t* scratch = nullptr;
};
NoAllocDevice g_noalloc_devices[64];

}  // namespace

extern "C" int bm_gemm_run_noalloc(const bm_gemm_desc* d, void* stream, uint32_t* device_status) {
  if (device_status) *device_status = 0;
  int rc = bm_gemm_check(d);
  if (rc != BM_OK) return rc;
  if (kNoAllocScratchPerCall > kNoAllocScratchBytes) return BM_ERR_SCRATCH_LIMIT;
  Resolved r;
  resolve(d, &r);
  const int v = pick_variant(d);

  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return BM_ERR_CUDA;
  if (device < 0 || device >= 64) return BM_ERR_CUDA;
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return BM_ERR_CUDA;
  if (major != 10 || minor != 0) return BM_ERR_DEVICE;

  // Once per device, with that device current: device address of the array.
  NoAllocDevice& nd = g_noalloc_devices[device];
  std::call_once(nd.once, [&nd] {
    void* p = nullptr;
    nd.err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    nd.scratch = static_cast<uint32_t*>(p);
  });
  if (nd.err != cudaSuccess || nd.scratch == nullptr) return BM_ERR_CUDA;

  // A handle-shaped parameter block on the stack (no allocation).
  bm_gemm_handle h;
  std::memset(&h, 0, sizeof(h));
  h.variant = v;
  h.nt = r.nt;
  h.device = device;
  h.cta_group = kVariants[v].cta_group;
  h.tile_m = 128 * h.cta_group;
  h.tile_n = kVariants[v].mma_n * kVariants[v].num_n;
  h.stages = kVariants[v].stages;
  const int rows_b = kVariants[v].mma_n / h.cta_group;  // B rows per CTA per MMA
  bool ok;
  if (r.nt) {
    ok = encode_2d(&h.tmap_a, d->a, d->m, d->k, r.lda, 64, 64, true) &&
         encode_2d(&h.tmap_b, d->b, d->n, d->k, r.ldb, 64, 64, true);
  } else {
    ok = encode_2d(&h.tmap_a, d->a, d->k, d->m, r.lda, 64, 128, true) &&
         encode_2d(&h.tmap_b, d->b, d->k, d->n, r.ldb, 64, static_cast<uint32_t>(rows_b), true);
  }
  ok = ok && encode_2d(&h.tmap_c, d->c, d->m, d->n, r.ldc, 32, 32, false);
  if (!ok) return BM_ERR_CUDA;

  int max_clusters = 0, smem = 0;
  cudaError_t e = cudaErrorInvalidValue;
  switch (v * 2 + (r.nt ? 1 : 0)) {
#define BM_NOALLOC_CASE(VID, CG, BN, NN, ST)                                           \
  case VID * 2 + 0:                                                                    \
    e = geometry<CG, BN, NN, ST, false>(device, sms, VID, &max_clusters, &smem);       \
    h.launch = &launch_variant<CG, BN, NN, ST, false>;                                 \
    break;                                                                             \
  case VID * 2 + 1:                                                                    \
    e = geometry<CG, BN, NN, ST, true>(device, sms, VID, &max_clusters, &smem);        \
    h.launch = &launch_variant<CG, BN, NN, ST, true>;                                  \
    break;
    BM_FOR_EACH_VARIANT(BM_NOALLOC_CASE)
#undef BM_NOALLOC_CASE
    default: break;
  }
  if (e != cudaSuccess || max_clusters <= 0) return BM_ERR_CUDA;
  h.smem_bytes = smem;

  GemmParams& p = h.params;
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.tiles_m = (d->m + h.tile_m - 1) / h.tile_m;
  p.tiles_n = (d->n + h.tile_n - 1) / h.tile_n;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (d->k + 63) / 64;
  p.group_m = 8;
  p.timeout_ns = kDefaultTimeoutNs;
  p.debug = 0;
  p.stats = nullptr;
  p.status = nd.scratch;
  p.dp_tiles = p.num_tiles;  // whole tiles, one wave after another
  p.tail_parts = 0;
  p.tail_clusters = 0;
  const int clusters = p.num_tiles < max_clusters ? p.num_tiles : max_clusters;
  h.grid = clusters * h.cta_group;

  // The error word must start at zero; the array keeps the previous call's
  // contents otherwise. Ordered before the kernel on the same stream.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(nd.scratch, 0, kNoAllocScratchPerCall, s) != cudaSuccess) return BM_ERR_CUDA;
  if (h.launch(&h, s) != cudaSuccess) return BM_ERR_CUDA;
  if (device_status) {
    uint32_t bits = 0;
    if (cudaMemcpyAsync(&bits, nd.scratch, sizeof(bits), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return BM_ERR_CUDA;
    *device_status = bits;
    if (bits) return BM_ERR_DEVICE_TIMEOUT;
  }
  return BM_OK;
}
