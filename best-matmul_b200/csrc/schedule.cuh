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
// Memory-bound skinny problems (M <= 128, 1-CTA tiles) with fewer tiles than
// SMs instead split K: the tiles' k-blocks are divided evenly over all SMs
// (stream-K), so that every SM keeps loads in flight; partial tiles meet in an
// FP32 workspace. A piece that starts after k-block 0 is a contributor (writes
// its partial, raises its flags); the piece holding k-block 0 of a tile is its
// owner (waits for the flags, adds the partials in increasing k order, stores).
// Every cluster's range is contiguous, so a contributor piece is always a
// cluster's first piece of the split and an owner piece its last: owners wait
// only on work their contributors ran first, contributors never wait, and the
// hand-off cannot deadlock while the grid is resident.
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

enum : int { kUnitFull = 0, kUnitOwner = 1, kUnitContrib = 2 };

// Columns [q0 * kSplitCols, (q0 + w) * kSplitCols) and k-blocks [kb0, kb1) of
// tile `tile`. kind: kUnitFull (store), kUnitOwner (add the partials of
// clusters [cluster + 1, contrib_end), store), kUnitContrib (write a partial).
struct WorkUnit {
  int tile, q0, w;
  int kb0, kb1, kind, contrib_end;
};

// Cluster c's K-split range: [sk_start(c), sk_start(c + 1)) in the split
// tiles' k-blocks, counted tile-major from tile dp_tiles.
template <class P>
BM_HD long long sk_start(const P& p, int cluster) {
  return static_cast<long long>(cluster) * p.sk_total / p.sk_clusters;
}

// P has: int k_blocks, dp_tiles, tail_parts, tail_clusters, sk_clusters;
// long long sk_total. After the whole tiles, either column parts of the tail
// tiles (tail_parts > 0: numbered tile-major, cluster c < tail_clusters takes
// [c * Q / C, (c + 1) * Q / C)) or K-split pieces (sk_clusters > 0).
template <int kParts>
struct WorkIter {
  int next_tile, stride, cluster;
  long long g, g_end;

  template <class P>
  BM_HD WorkIter(const P& p, int cluster_id, int num_clusters)
      : next_tile(cluster_id), stride(num_clusters), cluster(cluster_id), g(0), g_end(0) {
    if (p.sk_clusters > 0) {
      if (cluster_id < p.sk_clusters) {
        g = sk_start(p, cluster_id);
        g_end = sk_start(p, cluster_id + 1);
      }
    } else if (cluster_id < p.tail_clusters) {
      g = static_cast<long long>(cluster_id) * p.tail_parts / p.tail_clusters;
      g_end = static_cast<long long>(cluster_id + 1) * p.tail_parts / p.tail_clusters;
    }
  }

  // True when next() has nothing left to return.
  template <class P>
  BM_HD bool done(const P& p) const {
    return next_tile >= p.dp_tiles && g >= g_end;
  }

  template <class P>
  BM_HD bool next(const P& p, WorkUnit& u) {
    u.kb0 = 0;
    u.kb1 = p.k_blocks;
    u.kind = kUnitFull;
    u.contrib_end = 0;
    if (next_tile < p.dp_tiles) {
      u.tile = next_tile;
      u.q0 = 0;
      u.w = kParts;
      next_tile += stride;
      return true;
    }
    if (g >= g_end) return false;
    if (p.sk_clusters > 0) {
      const int kb = p.k_blocks;
      const int st = static_cast<int>(g / kb);
      const int k0 = static_cast<int>(g - static_cast<long long>(st) * kb);
      const long long left = g_end - g;
      const int k1 = (left < kb - k0) ? k0 + static_cast<int>(left) : kb;
      u.tile = p.dp_tiles + st;
      u.q0 = 0;
      u.w = kParts;
      u.kb0 = k0;
      u.kb1 = k1;
      if (k0 > 0) {
        u.kind = kUnitContrib;
      } else if (k1 < kb) {
        u.kind = kUnitOwner;
        const long long tile_end = static_cast<long long>(st + 1) * kb;
        int j = cluster + 1;
        while (j < p.sk_clusters && sk_start(p, j) < tile_end) ++j;
        u.contrib_end = j;
      }
      g += k1 - k0;
      return true;
    }
    const int t = static_cast<int>(g / kParts);
    const int q0 = static_cast<int>(g - static_cast<long long>(t) * kParts);
    const int left = static_cast<int>(g_end - g);
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
  int sk_clusters;    // clusters sharing the K range of tiles [dp_tiles, tiles) (0: none)
  long long sk_total; // k-blocks of those tiles
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
  pl.sk_clusters = 0;
  pl.sk_total = 0;
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

// K split of a memory-bound grid: when a problem has fewer tiles than
// clusters, every cluster takes an even share of all tiles' k-blocks, so all
// of them stream operands. Each piece is at least min_kb k-blocks (pieces of
// one tile stay few). Leaves the plan unchanged otherwise.
inline Plan plan_k_split(int tiles, int k_blocks, int clusters, int min_kb) {
  Plan pl = plan_schedule(tiles, 1, clusters, 0);
  if (tiles <= 0 || clusters <= 0 || k_blocks <= 0 || tiles >= clusters) return pl;
  const long long total = static_cast<long long>(tiles) * k_blocks;
  long long skc = clusters;
  const int min_piece = min_kb > 1 ? min_kb : 1;  // every cluster gets k-blocks
  if (total / min_piece < skc) skc = total / min_piece;
  if (skc <= tiles) return pl;  // no more clusters busy than whole tiles give
  pl.dp_tiles = 0;
  pl.sk_clusters = static_cast<int>(skc);
  pl.sk_total = total;
  pl.grid_clusters = static_cast<int>(skc);
  pl.est = static_cast<double>(total) / static_cast<double>(skc) / k_blocks;
  return pl;
}

}  // namespace bm
