// Work schedule of the persistent GEMM grid: which tiles, and which column
// ranges of them, each cluster computes and in which order.
//
// The reference launches one CTA per output tile (grid = tiles_m x tiles_n,
// kernels/detail/tma_wgmma_adapter.cuh:96-113), so its last wave is partly
// idle whenever the tile count is not a multiple of the CTAs that fit at once.
// Here the persistent grid walks whole tiles in full waves; when the tiles
// left over for the last wave are at most half the clusters, they are cut into
// column halves (256 columns, one N = 256 MMA per K step instead of two) so
// that twice as many clusters share them and the last wave takes half a
// tile-time. Narrower pieces do not pay on B200: an N = 128 MMA of the pair
// costs about as much as an N = 256 one. Every output element is still one
// MMA chain over all of K in the same order, so a split launch gives the same
// bits as a whole-tile launch; no partial sums, workspace or inter-CTA waits.
//
// Plain C++ when not compiled by nvcc: tests/native/schedule_check.cpp runs
// the same planner and iterator on the CPU.
#pragma once

#if defined(__CUDACC__)
#define BM_HD __host__ __device__ __forceinline__
#else
#define BM_HD inline
#endif

namespace bm {

constexpr int kSplitCols = 256;  // column granularity of split tiles

// Columns [q0 * kSplitCols, (q0 + w) * kSplitCols) of tile `tile`, all of K.
struct WorkUnit {
  int tile, q0, w;
};

// P has: int dp_tiles, tail_parts, tail_clusters. Column parts of the tail
// tiles (tiles dp_tiles, dp_tiles + 1, ...) are numbered tile-major; cluster c
// (c < tail_clusters) takes [c * Q / C, (c + 1) * Q / C), Q = tail_parts,
// C = tail_clusters.
template <int kParts>
struct WorkIter {
  int next_tile, stride;
  int g, g_end;

  template <class P>
  BM_HD WorkIter(const P& p, int cluster, int num_clusters)
      : next_tile(cluster), stride(num_clusters), g(0), g_end(0) {
    if (cluster < p.tail_clusters) {
      g = static_cast<int>(static_cast<long long>(cluster) * p.tail_parts / p.tail_clusters);
      g_end = static_cast<int>(static_cast<long long>(cluster + 1) * p.tail_parts / p.tail_clusters);
    }
  }

  // True when next() has nothing left to return.
  template <class P>
  BM_HD bool done(const P& p) const {
    return next_tile >= p.dp_tiles && g >= g_end;
  }

  template <class P>
  BM_HD bool next(const P& p, WorkUnit& u) {
    if (next_tile < p.dp_tiles) {
      u.tile = next_tile;
      u.q0 = 0;
      u.w = kParts;
      next_tile += stride;
      return true;
    }
    if (g >= g_end) return false;
    const int t = g / kParts;
    const int q0 = g - t * kParts;
    const int left = g_end - g;
    const int w = (left < kParts - q0) ? left : kParts - q0;
    u.tile = p.dp_tiles + t;
    u.q0 = q0;
    u.w = w;
    g += w;
    return true;
  }
};

// ------------------------------------------------------------ host planner
struct Plan {
  int dp_tiles;       // whole tiles, in full waves
  int tail_parts;     // column parts of the remaining tiles (0: no split)
  int tail_clusters;  // clusters sharing them
  int grid_clusters;  // clusters to launch
  double est;         // estimated time in whole-tile mainloops
};

// tiles: tile count; parts: column parts per tile (1 = cannot split);
// clusters: resident clusters; split: 0 = whole tiles only, 1 = split the
// tail when that shortens it.
// With rem = tiles mod clusters tiles left for the last wave, the rem * q
// parts go to clusters in runs of r = ceil(rem * q / clusters) parts (the
// tail then takes r / q of a tile-time instead of one), over just
// ceil(rem * q / r) clusters so that every run but the last has exactly r.
inline Plan plan_schedule(int tiles, int parts, int clusters, int split) {
  Plan pl;
  pl.dp_tiles = tiles;
  pl.tail_parts = 0;
  pl.tail_clusters = 0;
  pl.grid_clusters = tiles < clusters ? tiles : clusters;
  pl.est = clusters > 0 ? static_cast<double>((tiles + clusters - 1) / clusters) : 0.0;
  if (!split || parts <= 1 || tiles <= 0 || clusters <= 0) return pl;
  const int rem = tiles % clusters;
  if (rem == 0) return pl;
  const int q_total = rem * parts;
  const int run = (q_total + clusters - 1) / clusters;
  if (run >= parts) return pl;  // no shorter than a whole tile
  pl.dp_tiles = tiles - rem;
  pl.tail_parts = q_total;
  pl.tail_clusters = (q_total + run - 1) / run;
  pl.grid_clusters = pl.dp_tiles > 0 ? clusters : pl.tail_clusters;
  pl.est = static_cast<double>(tiles / clusters) + static_cast<double>(run) / parts;
  return pl;
}

}  // namespace bm
