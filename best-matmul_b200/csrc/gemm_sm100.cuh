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
//   warps 2..5  epilogue: TMEM -> registers -> FP16 -> smem -> TMA store,
//               overlapped with the next tile's mainloop via two TMEM
//               accumulator buffers
//
// kCtaGroup == 2 runs each tile on a CTA pair (cluster 2x1) with
// tcgen05.mma.cta_group::2: the pair computes a 256 x kBN tile, each CTA loads
// its own 128 rows of A and kBN/2 rows of B (no multicast), and each CTA's
// TMEM holds its 128 output rows.
//
// Every wait is bounded (ptx::bm_wait); on expiry the CTA records an error
// code in the device status word, tells its other roles to stop, drains its
// own in-flight work with bounded waits, frees TMEM and returns.
#pragma once

#include <cuda_fp16.h>
#include "ptx_sm100.cuh"

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
  int tiles_m, tiles_n;  // tile grid in units of (kTileM x kBN)
  int num_tiles;
  int k_blocks;          // ceil(k / 64)
  int group_m;           // rasterization: tiles of group_m M-blocks share B in L2
  uint32_t* status;      // device error word (OR of kStatus* bits)
  uint64_t timeout_ns;   // bound on every mbarrier wait
  uint32_t debug;        // kDebug* flags; 0 in production
};

template <int kCtaGroup, int kBN, int kStages, bool kMnMajor>
struct GemmConfig {
  static constexpr int kThreads = 192;
  static constexpr int kBK = 64;                       // one 128-byte swizzle row of FP16
  static constexpr int kRowsA = 128;                   // A rows per CTA (TMEM lanes)
  static constexpr int kTileM = 128 * kCtaGroup;       // output rows per tile
  static constexpr int kRowsB = kBN / kCtaGroup;       // B rows loaded per CTA
  static constexpr int kMmaM = 128 * kCtaGroup;
  static constexpr int kBytesA = kRowsA * kBK * 2;     // 16 KB
  static constexpr int kBytesB = kRowsB * kBK * 2;
  static constexpr int kStageBytes = kBytesA + kBytesB;
  static constexpr int kEpiBoxRows = 32;               // one warp's TMEM lane quarter
  static constexpr int kEpiBoxCols = 32;
  static constexpr int kEpiBufBytes = kEpiBoxRows * kEpiBoxCols * 2;  // 2 KB
  static constexpr int kEpiBytes = 4 * 2 * kEpiBufBytes;              // 4 warps x 2 buffers
  static constexpr int kTmemCols = 2 * kBN;            // two accumulator buffers
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

  static_assert(kBN % 64 == 0 && kBN <= 256, "kBN must be a multiple of 64, at most 256");
  static_assert(kRowsB % 64 == 0, "B rows per CTA must be a multiple of 64");
  static_assert(kTmemCols <= 512, "two accumulators must fit in TMEM");
  static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation must be a power of 2");
  static_assert(kBytesA % 1024 == 0 && kBytesB % 1024 == 0, "stages keep 1 KB alignment");
  static_assert(kSmemBytes <= 232448, "shared memory budget (227 KB) exceeded");
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

template <int kCtaGroup, int kBN, int kStages, bool kMnMajor>
__global__ void __launch_bounds__(192, 1)
bm_gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmap_a,
                     const __grid_constant__ CUtensorMap tmap_b,
                     const __grid_constant__ CUtensorMap tmap_c, const GemmParams p) {
  using Cfg = GemmConfig<kCtaGroup, kBN, kStages, kMnMajor>;
  extern __shared__ uint8_t smem_raw[];

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
      ptx::mbar_init(tempty_bar(a), 4 * kCtaGroup);   // one arrive per epilogue warp
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
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (kCtaGroup == 2) ptx::cluster_sync();  // peer barriers initialised
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

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
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        const int m0 = mb * Cfg::kTileM + static_cast<int>(cta_rank) * Cfg::kRowsA;
        const int n0 = nb * kBN + static_cast<int>(cta_rank) * Cfg::kRowsB;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::bm_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kStatusProducerTimeout);
            ok = false;
            break;
          }
          const int k0 = kb * Cfg::kBK;
          const uint32_t a_dst = sA + stage * Cfg::kBytesA;
          const uint32_t b_dst = sB + stage * Cfg::kBytesB;
          if constexpr (kCtaGroup == 1) {
            const uint32_t fb = full_bar(stage);
            ptx::mbar_arrive_expect_tx(fb, Cfg::kStageBytes);
            if constexpr (kMnMajor) {
              ptx::tma_load_2d(a_dst, &tmap_a, fb, m0, k0);
              ptx::tma_load_2d(a_dst + 8192, &tmap_a, fb, m0 + 64, k0);
#pragma unroll
              for (int j = 0; j < Cfg::kRowsB / 64; ++j)
                ptx::tma_load_2d(b_dst + 8192 * j, &tmap_b, fb, n0 + 64 * j, k0);
            } else {
              ptx::tma_load_2d(a_dst, &tmap_a, fb, k0, m0);
              ptx::tma_load_2d(b_dst, &tmap_b, fb, k0, n0);
            }
          } else {
            const uint32_t fb_leader = ptx::mapa(full_bar(stage), 0);
            if (leader) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * Cfg::kStageBytes);
            if constexpr (kMnMajor) {
              ptx::tma_load_2d_pair(a_dst, &tmap_a, fb_leader, m0, k0);
              ptx::tma_load_2d_pair(a_dst + 8192, &tmap_a, fb_leader, m0 + 64, k0);
#pragma unroll
              for (int j = 0; j < Cfg::kRowsB / 64; ++j)
                ptx::tma_load_2d_pair(b_dst + 8192 * j, &tmap_b, fb_leader, n0 + 64 * j, k0);
            } else {
              ptx::tma_load_2d_pair(a_dst, &tmap_a, fb_leader, k0, m0);
              ptx::tma_load_2d_pair(b_dst, &tmap_b, fb_leader, k0, n0);
            }
          }
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
      for (int tile = cluster_id; tile < p.num_tiles && ok; tile += num_clusters) {
        if (!ptx::bm_wait(tempty_bar(acc), acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
          fail(kStatusMmaTimeout);
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ptx::bm_wait(full_bar(stage), phase, p.timeout_ns, abort_flag)) {
            fail(kStatusMmaTimeout);
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_base = sA + stage * Cfg::kBytesA;
          const uint32_t b_base = sB + stage * Cfg::kBytesB;
#pragma unroll
          for (int ks = 0; ks < Cfg::kBK / 16; ++ks) {
            uint64_t a_desc, b_desc;
            if constexpr (kMnMajor) {
              // 64 MN-elements per 128-byte row, one row per k; 8-row swizzle
              // atoms are 1 KB apart (SBO); 64-element MN chunks 8 KB apart
              // (LBO). One K=16 step covers 16 rows = 2 KB.
              a_desc = ptx::smem_desc_sw128(a_base + ks * 2048, 8192, 1024);
              b_desc = ptx::smem_desc_sw128(b_base + ks * 2048, 8192, 1024);
            } else {
              // One 128-byte row (64 k) per M/N row; 8-row atoms 1 KB apart.
              // One K=16 step advances 32 bytes inside the swizzled row.
              a_desc = ptx::smem_desc_sw128(a_base + ks * 32, 16, 1024);
              b_desc = ptx::smem_desc_sw128(b_base + ks * 32, 16, 1024);
            }
            ptx::mma_f16<kCtaGroup>(d_tmem, a_desc, b_desc, Cfg::kIdesc,
                                    (kb > 0 || ks > 0) ? 1u : 0u);
          }
          // Free this stage in every CTA that loaded into it.
          ptx::mma_commit<kCtaGroup>(empty_bar(stage));
          if constexpr (kCtaGroup == 2) ptx::mma_commit<kCtaGroup>(ptx::mapa(empty_bar(stage), peer));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // Accumulator complete -> both CTAs' epilogues.
        ptx::mma_commit<kCtaGroup>(tfull_bar(acc));
        if constexpr (kCtaGroup == 2) ptx::mma_commit<kCtaGroup>(ptx::mapa(tfull_bar(acc), peer));
        if (++acc == 2) {
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
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int ew = warp - 2;       // epilogue warp index 0..3 (staging buffers)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tempty_leader0 = (kCtaGroup == 2) ? ptx::mapa(tempty_bar(0), 0) : tempty_bar(0);
    const uint32_t tempty_leader1 = (kCtaGroup == 2) ? ptx::mapa(tempty_bar(1), 0) : tempty_bar(1);
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
    int chunk = 0;  // running chunk count -> staging buffer parity
    for (int tile = cluster_id; tile < p.num_tiles && ok; tile += num_clusters) {
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      if (!ptx::bm_wait(tfull_bar(acc), acc_phase, p.timeout_ns, abort_flag)) {
        if (lane == 0) fail(kStatusEpilogueTimeout);
        break;
      }
      ptx::tc_fence_after();
      const int row0 = mb * Cfg::kTileM + static_cast<int>(cta_rank) * 128 + quarter * 32;
      const int col0 = nb * kBN;
      const uint32_t t_acc = tmem_base + lane_base + static_cast<uint32_t>(acc * kBN);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c, ++chunk) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(c * 32), r);
        ptx::tmem_wait_ld();
        if (c == kBN / 32 - 1) {
          // All of this warp's TMEM reads for the tile are done: hand the
          // accumulator back to the MMA issuer before the stores.
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            const uint32_t tb = acc ? tempty_leader1 : tempty_leader0;
            if constexpr (kCtaGroup == 2) ptx::mbar_arrive_cluster(tb);
            else ptx::mbar_arrive(tb);
          }
        }
        const uint32_t buf = sEpi + static_cast<uint32_t>((ew * 2 + (chunk & 1)) * Cfg::kEpiBufBytes);
        if (lane == 0) ptx::bulk_wait_group_read<1>();  // buffer from 2 chunks ago is free
        __syncwarp();
        __half* hb = reinterpret_cast<__half*>(smem + (buf - base));
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          hb[j * 32 + lane] = __float2half_rn(__uint_as_float(r[j]));
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_2d(&tmap_c, buf, row0, col0 + c * 32);
          ptx::bulk_commit_group();
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (kCtaGroup == 2) ptx::cluster_sync();  // peer done with our smem/barriers
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc<kCtaGroup>(tmem_base, Cfg::kTmemCols);
}

}  // namespace bm
