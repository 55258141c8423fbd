// Persistent, warp-specialized FP16 GEMM for sm_100a (B200).
//
//   C(M,N) = A(M,K) * B(N,K)^T      FP16 in, FP32 accumulate (TMEM), FP16 out
//
// Layout contract (the reference's GemmProblem, host/common.cuh:43-76):
//   NT: a[m + k*lda], b[n + k*ldb]   (M / N contiguous -> "MN-major" operands)
//   TN: a[m*lda + k], b[n*ldb + k]   (K contiguous     -> "K-major"  operands)
//   C : c[m + n*ldc]                 (column-major, always)
//
// The reference's mainloop (kernels/wgmma_tma_fp16_warp_specialized_v4.cuh:109-190)
// is one output tile per CTA with register accumulators and a serialized
// epilogue. This kernel is organised around Blackwell's execution model instead:
//
//   warp 0      TMA producer: fills a kStages-deep shared-memory ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma into TMEM; owns TMEM
//   warps 2..9  epilogue: TMEM -> registers -> FP16 -> smem -> TMA store;
//               two warps per TMEM lane quarter, each draining half the columns
//
// Tile geometry (template parameters):
//   kCtaGroup  1: one CTA computes 128 rows; 2: a CTA pair (cluster 2x1) runs
//              tcgen05.mma.cta_group::2 and computes 256 rows, each CTA holding
//              its own 128 rows of A and half of every B block (no multicast).
//   kBN        N of one MMA instruction (128 or 256).
//   kNumN      MMAs per K step that share the same A tile (1 or 2): the tile
//              is kBN * kNumN wide, so every A byte brought on chip feeds
//              kNumN MMAs. kNumN = 2 with kBN = 256 fills all 512 TMEM columns.
// With room for two accumulators in TMEM (kAccStages = 2) the epilogue of tile
// i overlaps the mainloop of tile i+1. With one (the 256x512 pair tile) the
// epilogue reads the accumulator into packed FP16 registers and releases TMEM
// before storing, first columns [0, 256) then [256, 512), and the MMA issuer
// starts the next tile's first k-blocks on the half that is free first.
// Tiles are scheduled by schedule.cuh (whole tiles in full waves; a half-empty
// last wave in 256-column halves).
//
// Every wait is bounded (ptx::bm_wait); on expiry the CTA records an error
// code in the device status word, tells its other roles to stop, drains its
// own in-flight work with bounded waits, frees TMEM and returns.
#pragma once

#include <cuda_fp16.h>
#include "ptx_sm100.cuh"
#include "schedule.cuh"

namespace bm {

// Status bits written to the device status word.
enum : uint32_t {
  kStatusProducerTimeout = 1u << 0,
  kStatusMmaTimeout = 1u << 1,
  kStatusEpilogueTimeout = 1u << 2,
  kStatusDrainTimeout = 1u << 3,
  kStatusForcedWait = 1u << 4,  // the debug wait on a never-signalled barrier expired
};

// Debug flags (kernel parameter).
enum : uint32_t {
  kDebugEpilogueWaitsNever = 1u << 0,  // epilogue first waits on a barrier nothing signals
};

struct GemmParams {
  int m, n, k;
  int tiles_m, tiles_n;  // tile grid in units of (kTileM x kTileN)
  int num_tiles;
  int k_blocks;          // ceil(k / 64)
  int group_m;           // rasterization: tiles of group_m M-blocks share B in L2
  uint32_t* status;      // device error word (OR of kStatus* bits)
  uint64_t timeout_ns;   // bound on every mbarrier wait
  uint32_t debug;        // kDebug* flags; 0 in production
  unsigned long long* stats;  // per-CTA cycle counters; only read in BM_KERNEL_STATS builds
  // Schedule (schedule.cuh): tiles [0, dp_tiles) whole, cluster c taking c,
  // c + clusters, ...; then the column halves of tiles [dp_tiles,
  // num_tiles) split over clusters [0, tail_clusters) (tail_parts = 0:
  // nothing split).
  int dp_tiles;
  int tail_parts;
  int tail_clusters;
};

// Opt-in pipeline counters (build with -DBM_KERNEL_STATS): per CTA, cycles
// spent in each role's waits and a few timestamps, for diagnosing where the
// mainloop stalls. Product builds compile them out entirely.
enum StatSlot : int {
  kStatTotal = 0, kStatProdWait, kStatProdWaits, kStatMmaFullWait, kStatMmaFullWaits,
  kStatMmaTmemWait, kStatMmaTmemWaits, kStatEpiWait, kStatEpiWaits, kStatEpiBusy,
  kStatTiles, kStatKBlocks, kStatT0, kStatT1, kStatMmaFirst, kStatMmaLast,
  // per tile u < kStatUnits (kStatUnitFields slots each), %globaltimer ns:
  // MMA start, MMA end (last commit issued), epilogue start (accumulator
  // ready), TMEM released, epilogue end (stores issued); then the MMA
  // thread's cycles waiting for loaded stages during the tile, and its
  // clock64 cycles from MMA start to MMA end. Written straight to global
  // memory by the MMA thread and epilogue warp 2.
  kStatUnit0 = 16, kStatUnits = 6, kStatUnitFields = 7,
  kStatUnitCount = kStatUnit0 + kStatUnitFields * kStatUnits,
  // set-up, %globaltimer ns (warp 1): TMEM allocated, CTA barrier, cluster barrier
  kStatSetupAlloc, kStatSetupSync, kStatSetupCluster,
  kNumStats
};

#if defined(BM_KERNEL_STATS)
__device__ __forceinline__ bool stat_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                          const volatile uint32_t* abort_flag,
                                          unsigned long long& cycles, unsigned long long& count) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  const bool ok = ptx::bm_wait(bar, parity, timeout_ns, abort_flag);
  cycles += static_cast<unsigned long long>(clock64() - t0);
  count += 1;
  return ok;
}
#define BM_WAIT(bar, par, to, ab, CYC, CNT) stat_wait(bar, par, to, ab, st[CYC], st[CNT])
#define BM_STAT_PUT(slot, v) \
  do { if (p.stats) p.stats[static_cast<size_t>(blockIdx.x) * kNumStats + (slot)] = (v); } while (0)
#else
#define BM_WAIT(bar, par, to, ab, CYC, CNT) ptx::bm_wait(bar, par, to, ab)
#endif

constexpr int kEpiWarps = 8;                        // two per TMEM lane quarter
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;   // producer + MMA + epilogue warps

template <int kCtaGroup, int kBN, int kNumN, int kStages, bool kMnMajor>
struct GemmConfig {
  static constexpr int kThreads = kGemmThreads;
  static constexpr int kBK = 64;                        // one 128-byte swizzle row of FP16
  static constexpr int kRowsA = 128;                    // A rows per CTA (TMEM lanes)
  static constexpr int kTileM = 128 * kCtaGroup;        // output rows per tile
  static constexpr int kTileN = kBN * kNumN;            // output columns per tile
  static constexpr int kMmaM = 128 * kCtaGroup;
  static constexpr int kRowsBPerMma = kBN / kCtaGroup;  // B rows per CTA for one MMA
  static constexpr int kBytesA = kRowsA * kBK * 2;      // 16 KB
  static constexpr int kBytesBPerMma = kRowsBPerMma * kBK * 2;
  static constexpr int kBytesB = kBytesBPerMma * kNumN;
  static constexpr int kStageBytes = kBytesA + kBytesB;
  static constexpr int kAccCols = kBN * kNumN;          // TMEM columns of one accumulator
  static constexpr int kAccStages = (2 * kAccCols <= 512) ? 2 : 1;
  static constexpr int kTmemCols = kAccCols * kAccStages;
  static constexpr int kChunks = kAccCols / 32;         // epilogue chunks of 32 columns
  static constexpr int kChunksPerWarp = kChunks / 2;    // each lane quarter has two warps
  static constexpr int kEpiBoxRows = 32;                // one warp's TMEM lane quarter
  static constexpr int kEpiBoxCols = 32;
  static constexpr int kEpiBufBytes = kEpiBoxRows * kEpiBoxCols * 2;  // 2 KB
  static constexpr int kEpiBytes = kEpiWarps * 2 * kEpiBufBytes;      // 2 buffers per warp
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kBytesA;
  static constexpr int kOffEpi = kOffB + kStages * kBytesB;
  static constexpr int kOffBar = kOffEpi + kEpiBytes;
  // barriers: full[S], empty[S], tmem_full[2], tmem_empty[2], drain, never
  static constexpr int kNumBars = 2 * kStages + 6;
  static constexpr int kOffTmemSlot = kOffBar + 8 * kNumBars;
  static constexpr int kOffAbort = kOffTmemSlot + 4;
  static constexpr int kSmemBytes = kOffAbort + 4 + 1024;  // + alignment slack
  static constexpr uint32_t kIdesc = make_idesc_f16_f32(kMmaM, kBN, kMnMajor);
  // Column parts per tile, and whether leftover tiles may be computed in
  // parts (the 256x512 pair tile: a 256-column half is one N = 256 MMA per
  // K step instead of two).
  static constexpr bool kTailSplit = (kCtaGroup == 2 && kNumN == 2 && kBN == 256);
  // One accumulator of 512 columns whose halves the epilogue releases one
  // after the other: tempty_bar(0) frees columns [0, 256), tempty_bar(1)
  // columns [256, 512) (kAccStages == 1 leaves the second barrier free).
  static constexpr bool kHalfRelease = kTailSplit;
  static_assert(!kHalfRelease || (kAccStages == 1 && kTileN == 512), "half release layout");
  static constexpr int kParts = kTailSplit ? kTileN / kSplitCols : 1;

  static_assert(kBN == 128 || kBN == 256, "kBN must be 128 or 256");
  static_assert(kNumN == 1 || kNumN == 2, "kNumN must be 1 or 2");
  static_assert(kRowsBPerMma % 64 == 0, "B rows per CTA and MMA must be a multiple of 64");
  static_assert(kTmemCols <= 512, "accumulators must fit in TMEM");
  static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation must be a power of 2");
  static_assert(kChunksPerWarp % 2 == 0, "each epilogue warp processes chunks in pairs");
  static_assert(kBytesA % 1024 == 0 && kBytesBPerMma % 1024 == 0, "stages keep 1 KB alignment");
  static_assert(kSmemBytes <= 232448, "shared memory budget (227 KB) exceeded");
  static_assert(kStages * kStageBytes >= kEpiWarps * kChunksPerWarp * kEpiBufBytes,
                "the last tile's epilogue stages every chunk in the free mainloop stages");
};

// Epilogue ownership (shared with the host-side mapping check): epilogue warp
// `warp` (2..9) reads TMEM lane quarter warp % 4; the two warps of a quarter
// share a unit's 32-column chunks, cpw each, the warp's cc-th chunk being
// epi_chunk(warp, cc, cpw, half_order). With half_order (the 256x512 pair
// tile) both warps first take chunks of columns [0, 256) and then of
// [256, 512), so that the first TMEM half can be released early. In chunk
// `chunk`, step i (0..15), lane `lane` stores one 32-bit word: two consecutive
// rows of one column of the CTA's 128-row tile.
struct EpiCoord {
  int row;  // first of the two rows (row, row + 1) within the CTA's 128 rows
  int col;  // column within the tile
};
__host__ __device__ constexpr int epi_quarter(int warp) { return warp & 3; }
__host__ __device__ constexpr bool epi_half_order(int tile_n) { return tile_n == 512; }
__host__ __device__ constexpr int epi_chunk(int warp, int cc, int cpw, bool half_order) {
  return half_order ? (cc / 4) * 8 + ((warp - 2) / 4) * 4 + cc % 4 : ((warp - 2) / 4) * cpw + cc;
}
__host__ __device__ constexpr EpiCoord epi_word_coord(int warp, int lane, int chunk, int i) {
  return EpiCoord{epi_quarter(warp) * 32 + (lane & ~1), chunk * 32 + 2 * i + (lane & 1)};
}

template <int N>
struct IntTag {
  static constexpr int value = N;
};

// Tile index -> (m block, n block). Tiles are walked in bands of group_m
// M-blocks so that concurrently running CTAs share B (and A) tiles in L2.
__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mb, int& nb) {
  const int per_group = p.group_m * p.tiles_n;
  const int group = tile / per_group;
  const int first_m = group * p.group_m;
  const int rows = min(p.tiles_m - first_m, p.group_m);
  const int in_group = tile - group * per_group;
  mb = first_m + in_group % rows;
  nb = in_group / rows;
}

template <int kCtaGroup, int kBN, int kNumN, int kStages, bool kMnMajor>
__global__ void __launch_bounds__(kGemmThreads, 1)
bm_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_c, const GemmParams p) {
  using Cfg = GemmConfig<kCtaGroup, kBN, kNumN, kStages, kMnMajor>;
  extern __shared__ uint8_t smem_raw[];

#if defined(BM_KERNEL_STATS)
  const unsigned long long g_entry = ptx::globaltimer_ns();
#endif
  // 1 KB alignment for the 128-byte-swizzled tiles. Both CTAs of a pair run
  // the same code, so the offsets (and hence the MMA descriptors) agree.
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta_rank = (kCtaGroup == 2) ? ptx::cluster_ctarank() : 0u;
  const bool leader = (cta_rank == 0);
  const int cluster_id = blockIdx.x / kCtaGroup;
  const int num_clusters = gridDim.x / kCtaGroup;

  const uint32_t sA = base + Cfg::kOffA;
  const uint32_t sB = base + Cfg::kOffB;
  const uint32_t sEpi = base + Cfg::kOffEpi;
  const uint32_t bar0 = base + Cfg::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * kStages + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * kStages + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kStages + 4);
  const uint32_t never_bar = bar0 + 8u * (2 * kStages + 5);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffTmemSlot);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + Cfg::kOffAbort);

  // ------------------------------------------------------------ set-up
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tmap_a);
    ptx::prefetch_tmap(&tmap_b);
    ptx::prefetch_tmap(&tmap_c);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(full_bar(s), 1);   // the (leader) producer's arrive.expect_tx
      ptx::mbar_init(empty_bar(s), 1);  // one tcgen05.commit per use
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(tfull_bar(a), 1);                // one tcgen05.commit per tile
      ptx::mbar_init(tempty_bar(a), kEpiWarps * kCtaGroup);  // one arrive per epilogue warp
    }
    ptx::mbar_init(drain_bar, 1);
    ptx::mbar_init(never_bar, 1);
    *abort_flag = 0u;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc<kCtaGroup>(ptx::smem_u32(tmem_slot), Cfg::kTmemCols);
    ptx::tmem_relinquish<kCtaGroup>();
  }
#if defined(BM_KERNEL_STATS)
  const unsigned long long g_alloc = ptx::globaltimer_ns();
#endif
  ptx::tc_fence_before();
  __syncthreads();
#if defined(BM_KERNEL_STATS)
  const unsigned long long g_sync = ptx::globaltimer_ns();
#endif
  if constexpr (kCtaGroup == 2) ptx::cluster_sync();  // peer barriers initialised
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touched only shared memory, TMEM and kernel parameters,
  // so it may overlap the previous kernel in the stream (launched with
  // programmatic stream serialization). Global memory (A, B, C, the status
  // word) is touched only after the previous grid has completed.
  ptx::griddep_wait();
  if (threadIdx.x == 0) ptx::griddep_launch_dependents();
#if defined(BM_KERNEL_STATS)
  unsigned long long st[kNumStats] = {};  // constant indices only: registers
  const long long t_begin = clock64();
  if (warp == 1 && lane == 0) {
    BM_STAT_PUT(kStatSetupAlloc, g_alloc);
    BM_STAT_PUT(kStatSetupSync, g_sync);
    BM_STAT_PUT(kStatSetupCluster, ptx::globaltimer_ns());
  }
  int unit_i = 0;
  unsigned long long unit_wait0 = 0;
#endif

  auto fail = [&](uint32_t bit) {
    *abort_flag = 1u;
    atomicOr(p.status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Every TMA box of k-block kb of unit w for this CTA:
      // f(is_b, byte offset in the stage's A or B part, tensor map, x, y).
      // Columns of the unit: n_unit from nbase; MMA j covers
      // [nbase + j*kBN, + nj), nj = min(n_unit - j*kBN, kBN) (<= 0: no MMA j),
      // and this CTA holds B rows [rank * nj / kCtaGroup, + nj / kCtaGroup).
      // MN-major (NT) tiles are 64-wide boxes 8 KB apart; K-major (TN) tiles
      // are one box per operand and MMA (whole boxes of kRowsBPerMma rows).
      auto unit_boxes = [&](const WorkUnit& w, int kb, auto&& f) {
        int mb, nb;
        tile_coords(w.tile, p, mb, nb);
        const int n_unit = Cfg::kTailSplit ? w.w * kSplitCols : Cfg::kTileN;
        const int nbase = nb * Cfg::kTileN + (Cfg::kTailSplit ? w.q0 * kSplitCols : 0);
        const int m0 = mb * Cfg::kTileM + static_cast<int>(cta_rank) * Cfg::kRowsA;
        const int k0 = kb * Cfg::kBK;
        if constexpr (kMnMajor) {
          f(false, 0u, &tmap_a, m0, k0);
          f(false, 8192u, &tmap_a, m0 + 64, k0);
        } else {
          f(false, 0u, &tmap_a, k0, m0);
        }
#pragma unroll
        for (int j = 0; j < kNumN; ++j) {
          const int nj = min(n_unit - j * kBN, kBN);
          if (nj <= 0) break;
          const int rows = nj / kCtaGroup;
          const int r0 = nbase + j * kBN + static_cast<int>(cta_rank) * rows;
          const uint32_t off = static_cast<uint32_t>(j * Cfg::kBytesBPerMma);
          if constexpr (kMnMajor) {
#pragma unroll
            for (int q = 0; q < Cfg::kRowsBPerMma / 64; ++q)
              if (64 * q < rows) f(true, off + 8192u * q, &tmap_b, r0 + 64 * q, k0);
          } else {
            f(true, off, &tmap_b, k0, r0);
          }
        }
      };
      WorkIter<Cfg::kParts> it(p, cluster_id, num_clusters);
      WorkUnit u;
      while (ok && it.next(p, u)) {
        // Bytes this CTA lands per stage for this unit.
        uint32_t stage_bytes = 0;
        unit_boxes(u, 0, [&](bool is_b, uint32_t, const CUtensorMap*, int, int) {
          stage_bytes += is_b ? (kMnMajor ? 8192u : static_cast<uint32_t>(Cfg::kBytesBPerMma))
                              : (kMnMajor ? 8192u : static_cast<uint32_t>(Cfg::kBytesA));
        });
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!BM_WAIT(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag, kStatProdWait, kStatProdWaits)) {
            fail(kStatusProducerTimeout);
            ok = false;
            break;
          }
          const uint32_t a_dst = sA + stage * Cfg::kBytesA;
          const uint32_t b_dst = sB + stage * Cfg::kBytesB;
          // Completion bytes go to this CTA's barrier (1 CTA) or the pair
          // leader's barrier (2 CTAs), which expects both CTAs' bytes.
          uint32_t fb;
          if constexpr (kCtaGroup == 1) {
            fb = full_bar(stage);
            ptx::mbar_arrive_expect_tx(fb, stage_bytes);
          } else {
            fb = ptx::mapa(full_bar(stage), 0);
            if (leader) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * stage_bytes);
          }
          unit_boxes(u, kb, [&](bool is_b, uint32_t off, const CUtensorMap* map, int x, int y) {
            const uint32_t dst = (is_b ? b_dst : a_dst) + off;
            if constexpr (kCtaGroup == 1) ptx::tma_load_2d(dst, map, fb, x, y);
            else ptx::tma_load_2d_pair(dst, map, fb, x, y);
          });
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every load this CTA issued must have landed before the CTA
      // can retire. On the normal path the MMA consumed them all already.
      if (!ok && (kCtaGroup == 1 || leader)) {
        for (int s = 0; s < kStages; ++s) {
          // The most recent use of stage s has parity phase^1 if s >= stage.
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          volatile uint32_t no_abort = 0u;
          if (!ptx::bm_wait(full_bar(s), par, p.timeout_ns, &no_abort)) {
            atomicOr(p.status, kStatusDrainTimeout);
            break;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t peer = 1u;
      WorkIter<Cfg::kParts> it(p, cluster_id, num_clusters);
      WorkUnit u;
      while (ok && it.next(p, u)) {
        // N of MMA j for this unit (whole tiles: kBN each, compile-time).
        const int n_unit = Cfg::kTailSplit ? u.w * kSplitCols : Cfg::kTileN;
        const int n0 = Cfg::kTailSplit ? min(n_unit, kBN) : kBN;
        const int n1 = Cfg::kTailSplit ? n_unit - kBN : kBN;
        const uint32_t idesc0 = Cfg::kTailSplit ? make_idesc_f16_f32(Cfg::kMmaM, n0, kMnMajor) : Cfg::kIdesc;
        const uint32_t idesc1 =
            Cfg::kTailSplit ? make_idesc_f16_f32(Cfg::kMmaM, n1 > 0 ? n1 : kBN, kMnMajor) : Cfg::kIdesc;
        const int n_mma = (kNumN == 2 && n1 > 0) ? 2 : 1;
        if (!BM_WAIT(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, abort_flag, kStatMmaTmemWait, kStatMmaTmemWaits)) {
          fail(kStatusMmaTimeout);
          break;
        }
        ptx::tc_fence_after();
#if defined(BM_KERNEL_STATS)
        if (unit_i < kStatUnits) BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i, ptx::globaltimer_ns());
        unit_wait0 = st[kStatMmaFullWait];
        const long long unit_clk0 = clock64();
#endif
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
        // MMAs j in [jlo, jhi) of k-block kb from stage stg.
        auto issue = [&](int stg, int kb, int jlo, int jhi) {
          // Descriptors of the stage's first K step; later steps and MMA 1's B
          // only move the start address (bits 0-13, 16-byte units), which
          // never carries out: all of shared memory lies below 256 KB.
          const uint32_t lbo = kMnMajor ? 8192u : 16u;
          const uint64_t a_desc0 = ptx::smem_desc_sw128(sA + stg * Cfg::kBytesA, lbo, 1024);
          const uint64_t b_desc0 = ptx::smem_desc_sw128(sB + stg * Cfg::kBytesB, lbo, 1024);
          // Consecutive MMAs go to the same accumulator (all K steps of MMA j,
          // then of MMA j+1): alternating accumulators every MMA measured
          // ~5 % fewer tensor cycles per k-block on B200.
#pragma unroll
          for (int j = 0; j < kNumN; ++j) {
            if (j < jlo || j >= jhi || j >= n_mma) continue;
#pragma unroll
            for (int ks = 0; ks < Cfg::kBK / 16; ++ks) {
              // MN-major: 64 MN-elements per 128-byte row, one row per k; 8-row
              // swizzle atoms 1 KB apart (SBO); 64-element MN chunks 8 KB apart
              // (LBO); one K=16 step is 16 rows = 2 KB.
              // K-major: one 128-byte row (64 k) per M/N row; 8-row atoms 1 KB
              // apart; one K=16 step advances 32 bytes inside the swizzled row.
              const uint32_t koff = kMnMajor ? ks * 2048u : ks * 32u;
              const uint64_t a_desc = a_desc0 + (koff >> 4);
              const uint64_t b_desc = b_desc0 + ((j * Cfg::kBytesBPerMma + koff) >> 4);
#if defined(BM_KERNEL_STATS)
              if (st[kStatMmaFirst] == 0) st[kStatMmaFirst] = ptx::globaltimer_ns();
#endif
              ptx::mma_f16<kCtaGroup>(d_tmem + static_cast<uint32_t>(j * kBN), a_desc, b_desc,
                                      j == 0 ? idesc0 : idesc1, (kb > 0 || ks > 0) ? 1u : 0u);
            }
          }
        };
        // Free a stage in every CTA that loaded into it.
        auto release_stage = [&](int stg) {
          ptx::mma_commit<kCtaGroup>(empty_bar(stg));
          if constexpr (kCtaGroup == 2) ptx::mma_commit<kCtaGroup>(ptx::mapa(empty_bar(stg), peer));
#if defined(BM_KERNEL_STATS)
          st[kStatKBlocks] += 1;
#endif
        };
        int kb = 0;
        if constexpr (Cfg::kHalfRelease) {
          // The epilogue hands back TMEM columns [0, 256) first: run MMA 0 of
          // the first kStages k-blocks (already loaded while the previous
          // tile drained) into them, then, once [256, 512) is free too, MMA 1
          // of the same k-blocks, releasing each stage after both.
          const int pre = p.k_blocks < kStages ? p.k_blocks : kStages;
          const int stage0 = stage;
          for (; kb < pre; ++kb) {
            if (!BM_WAIT(full_bar(stage), phase, p.timeout_ns, abort_flag, kStatMmaFullWait, kStatMmaFullWaits)) {
              fail(kStatusMmaTimeout);
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue(stage, kb, 0, 1);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          if (!BM_WAIT(tempty_bar(1), acc_phase ^ 1u, p.timeout_ns, abort_flag, kStatMmaTmemWait, kStatMmaTmemWaits)) {
            fail(kStatusMmaTimeout);
            break;
          }
          ptx::tc_fence_after();
          int s2 = stage0;
          for (int k2 = 0; k2 < pre; ++k2) {
            issue(s2, k2, 1, kNumN);
            release_stage(s2);
            if (++s2 == kStages) s2 = 0;
          }
        }
        for (; kb < p.k_blocks; ++kb) {
          if (!BM_WAIT(full_bar(stage), phase, p.timeout_ns, abort_flag, kStatMmaFullWait, kStatMmaFullWaits)) {
            fail(kStatusMmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue(stage, kb, 0, kNumN);
          release_stage(stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // Accumulator complete -> both CTAs' epilogues.
        ptx::mma_commit<kCtaGroup>(tfull_bar(acc));
        if constexpr (kCtaGroup == 2) ptx::mma_commit<kCtaGroup>(ptx::mapa(tfull_bar(acc), peer));
#if defined(BM_KERNEL_STATS)
        if (unit_i < kStatUnits) {
          BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 1, ptx::globaltimer_ns());
          BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 5, st[kStatMmaFullWait] - unit_wait0);
          BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 6,
                      static_cast<unsigned long long>(clock64() - unit_clk0));
        }
        ++unit_i;
        BM_STAT_PUT(kStatUnitCount, static_cast<unsigned long long>(unit_i));
#endif
        if (++acc == Cfg::kAccStages) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: wait until every MMA this thread issued has completed so
      // that TMEM can be released and shared memory can retire.
      ptx::mma_commit<kCtaGroup>(drain_bar);
      volatile uint32_t no_abort = 0u;
      if (!ptx::bm_wait(drain_bar, 0u, p.timeout_ns, &no_abort)) {
        atomicOr(p.status, kStatusDrainTimeout);
      }
#if defined(BM_KERNEL_STATS)
      st[kStatMmaLast] = ptx::globaltimer_ns();
#endif
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ epilogue
    const int quarter = epi_quarter(warp);  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int ew = warp - 2;                // epilogue warp index 0..7 (staging buffers)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tempty_leader0 = (kCtaGroup == 2) ? ptx::mapa(tempty_bar(0), 0) : tempty_bar(0);
    const uint32_t tempty_leader1 = (kCtaGroup == 2) ? ptx::mapa(tempty_bar(1), 0) : tempty_bar(1);
    const bool odd = (lane & 1) != 0;
    bool ok = true;
    if (p.debug & kDebugEpilogueWaitsNever) {
      // Fault-injection hook for tests: nothing ever arrives on never_bar,
      // so this wait must expire and report, never hang.
      volatile uint32_t no_abort = 0u;
      if (!ptx::bm_wait(never_bar, 0u, p.timeout_ns, &no_abort)) {
        if (lane == 0) fail(kStatusForcedWait);
        ok = false;
      }
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    int chunk_count = 0;  // running chunk count -> staging buffer parity

    // Convert one 32x32 chunk (this warp's 32 rows x 32 columns) to FP16 and
    // store it with one TMA box. Lane pairs swap halves so that each lane
    // writes one 32-bit word holding two consecutive rows of one column:
    // column-major C, conflict-free shared-memory stores.
    // Two FP32 values of one row (columns 2i, 2i+1) -> one word of FP16 pairs
    // laid out for column-major C: lane pairs swap halves so that the even
    // lane holds rows (lane, lane+1) of column 2i and the odd lane the same
    // rows of column 2i+1. Each value is rounded to FP16 on its own (round to
    // nearest even).
    auto pack_pair = [&](uint32_t c0v, uint32_t c1v) -> uint32_t {
      const __half2 own2 = __floats2half2_rn(__uint_as_float(c0v), __uint_as_float(c1v));
      const uint32_t own = *reinterpret_cast<const uint32_t*>(&own2);
      const uint32_t other = __shfl_xor_sync(0xffffffffu, own, 1);
      return odd ? __byte_perm(other, own, 0x7632) : __byte_perm(own, other, 0x5410);
    };

    // Stage one packed 32x32 chunk in shared memory and store it with one TMA
    // box. `big`: the CTA's last unit, whose mainloop stages are all consumed,
    // so every chunk of the warp (index `slot` among its chunks) gets its own
    // 2 KB of the stage area and nothing waits; otherwise two 2 KB buffers per
    // warp alternate.
    auto stage_store = [&](const uint32_t (&hw)[16], int row0, int col0, int chunk, bool big,
                           int slot) {
      uint32_t buf;
      if (big) {
        buf = sA + static_cast<uint32_t>((ew * Cfg::kChunksPerWarp + slot) * Cfg::kEpiBufBytes);
      } else {
        buf = sEpi + static_cast<uint32_t>((ew * 2 + (chunk_count & 1)) * Cfg::kEpiBufBytes);
        ++chunk_count;
        if (lane == 0) ptx::bulk_wait_group_read<1>();  // buffer from 2 chunks ago is free
        __syncwarp();
      }
      uint32_t* wb = reinterpret_cast<uint32_t*>(smem + (buf - base));
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // the 32x32 box is column-major: 16 words (32 rows) per column
        const EpiCoord e = epi_word_coord(warp, lane, chunk, i);
        wb[(e.col - chunk * 32) * 16 + ((e.row - quarter * 32) >> 1)] = hw[i];
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        ptx::tma_store_2d(&tmap_c, buf, row0, col0 + chunk * 32);
        ptx::bulk_commit_group();
      }
    };

    WorkIter<Cfg::kParts> it(p, cluster_id, num_clusters);
    WorkUnit u;
    while (ok && it.next(p, u)) {
      int mb, nb;
      tile_coords(u.tile, p, mb, nb);
      // This warp's chunks of the unit: the unit's n_unit / 32 chunks are
      // split in two halves between the two warps of each lane quarter.
      const int cpw = Cfg::kTailSplit ? u.w * (kSplitCols / 64) : Cfg::kChunksPerWarp;
      if (!BM_WAIT(tfull_bar(acc), acc_phase, p.timeout_ns, abort_flag, kStatEpiWait, kStatEpiWaits)) {
        if (lane == 0) fail(kStatusEpilogueTimeout);
        break;
      }
      ptx::tc_fence_after();
#if defined(BM_KERNEL_STATS)
      const long long t_epi = clock64();
      const bool put = warp == 2 && lane == 0 && unit_i < kStatUnits;
      if (put) BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 2, ptx::globaltimer_ns());
#endif
      const int row0 = mb * Cfg::kTileM + static_cast<int>(cta_rank) * 128 + quarter * 32;
      const int col0 = nb * Cfg::kTileN + (Cfg::kTailSplit ? u.q0 * kSplitCols : 0);
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * Cfg::kAccCols);
      const bool last = it.done(p);

      const int halves = 2 * cpw;
      constexpr bool kHalfOrder = epi_half_order(Cfg::kTileN);
      auto chunk_of = [&](int cc) { return epi_chunk(warp, cc, cpw, kHalfOrder); };
      // Hand TMEM back to the MMA issuer once this warp's reads of it have
      // completed: the whole accumulator (barrier acc), or with kHalfRelease
      // columns [0, 256) (h = 0) and [256, 512) (h = 1) separately.
      auto arrive_tempty = [&](int h) {
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const uint32_t tb = h ? tempty_leader1 : tempty_leader0;
          if constexpr (kCtaGroup == 2) ptx::mbar_arrive_cluster(tb);
          else ptx::mbar_arrive(tb);
        }
      };
      auto release_tmem = [&]() {
        if constexpr (Cfg::kHalfRelease) arrive_tempty(1);
        else arrive_tempty(acc);
#if defined(BM_KERNEL_STATS)
        if (put) BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 3, ptx::globaltimer_ns());
#endif
      };
      if (last) {
        // No next tile waits for TMEM: store each chunk as soon as it is
        // packed, so TMEM reads and stores overlap (16-column TMEM loads,
        // double-buffered).
        uint32_t ra[16], rb[16];
        ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(chunk_of(0) * 32), ra);
        ptx::tmem_wait_ld();
#pragma unroll 1
        for (int h = 0; h < halves; h += 2) {
          uint32_t hc[16];
          const int ch = chunk_of(h / 2);
          ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(ch * 32 + 16), rb);
#pragma unroll
          for (int i = 0; i < 8; ++i) hc[i] = pack_pair(ra[2 * i], ra[2 * i + 1]);
          ptx::tmem_wait_ld();
          if (h + 2 < halves)
            ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(chunk_of(h / 2 + 1) * 32), ra);
#pragma unroll
          for (int i = 0; i < 8; ++i) hc[8 + i] = pack_pair(rb[2 * i], rb[2 * i + 1]);
          stage_store(hc, row0, col0, ch, true, h / 2);
          if (h + 2 < halves) ptx::tmem_wait_ld();
        }
        if constexpr (Cfg::kHalfRelease) arrive_tempty(0);
        release_tmem();
      } else {
        // Read this warp's whole share of the accumulator into registers as
        // packed FP16 (load h+1 while packing h), hand TMEM back to the MMA
        // issuer, then store: the stores overlap the next tile's mainloop
        // instead of holding TMEM. One fully unrolled copy per unit width.
        auto drain = [&](auto cpw_tag) {
          constexpr int kCpw = decltype(cpw_tag)::value;
          uint32_t hw[kCpw][16];
          uint32_t ra[16], rb[16];
          ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(chunk_of(0) * 32), ra);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2 * kCpw; h += 2) {
            ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(chunk_of(h / 2) * 32 + 16), rb);
#pragma unroll
            for (int i = 0; i < 8; ++i) hw[h / 2][i] = pack_pair(ra[2 * i], ra[2 * i + 1]);
            ptx::tmem_wait_ld();
            // With the half order, chunks 0..3 of this warp are its share of
            // TMEM columns [0, 256): hand those back before reading the rest.
            if constexpr (Cfg::kHalfRelease) {
              if (h / 2 == 3) arrive_tempty(0);
            }
            if (h + 2 < 2 * kCpw)
              ptx::tmem_ld_32x32b_x16(t_acc + static_cast<uint32_t>(chunk_of(h / 2 + 1) * 32), ra);
#pragma unroll
            for (int i = 0; i < 8; ++i) hw[h / 2][8 + i] = pack_pair(rb[2 * i], rb[2 * i + 1]);
            if (h + 2 < 2 * kCpw) ptx::tmem_wait_ld();
          }
          release_tmem();
#pragma unroll
          for (int cc = 0; cc < kCpw; ++cc) stage_store(hw[cc], row0, col0, chunk_of(cc), false, cc);
        };
        if constexpr (Cfg::kTailSplit) {
          static_assert(Cfg::kChunksPerWarp == 8 && kSplitCols == 256, "units of one or two halves");
          if (cpw == 4) drain(IntTag<4>{});
          else drain(IntTag<8>{});
        } else {
          drain(IntTag<Cfg::kChunksPerWarp>{});
        }
      }
#if defined(BM_KERNEL_STATS)
      st[kStatEpiBusy] += static_cast<unsigned long long>(clock64() - t_epi);
      st[kStatTiles] += 1;
      if (put) BM_STAT_PUT(kStatUnit0 + kStatUnitFields * unit_i + 4, ptx::globaltimer_ns());
      ++unit_i;
#endif
      if (++acc == Cfg::kAccStages) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

#if defined(BM_KERNEL_STATS)
  if (p.stats != nullptr && lane == 0) {
    st[kStatTotal] = static_cast<unsigned long long>(clock64() - t_begin);
    unsigned long long* out = p.stats + static_cast<size_t>(blockIdx.x) * kNumStats;
    // one writer per role: producer (warp 0), MMA (warp 1), first epilogue warp (warp 2)
    if (warp == 0) {
      out[kStatTotal] = st[kStatTotal];
      out[kStatProdWait] = st[kStatProdWait];
      out[kStatProdWaits] = st[kStatProdWaits];
    } else if (warp == 1) {
      out[kStatMmaFirst] = st[kStatMmaFirst];
      out[kStatMmaLast] = st[kStatMmaLast];
      out[kStatMmaFullWait] = st[kStatMmaFullWait];
      out[kStatMmaFullWaits] = st[kStatMmaFullWaits];
      out[kStatMmaTmemWait] = st[kStatMmaTmemWait];
      out[kStatMmaTmemWaits] = st[kStatMmaTmemWaits];
      out[kStatKBlocks] = st[kStatKBlocks];
    } else if (warp == 2) {
      out[kStatT0] = g_entry;
      out[kStatT1] = ptx::globaltimer_ns();
      out[kStatEpiWait] = st[kStatEpiWait];
      out[kStatEpiWaits] = st[kStatEpiWaits];
      out[kStatEpiBusy] = st[kStatEpiBusy];
      out[kStatTiles] = st[kStatTiles];
    }
  }
#endif

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (kCtaGroup == 2) ptx::cluster_sync();  // peer done with our smem/barriers
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc<kCtaGroup>(tmem_base, Cfg::kTmemCols);
}

}  // namespace bm
