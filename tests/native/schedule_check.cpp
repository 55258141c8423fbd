// CPU check of the GEMM grid schedule (best-matmul_b200/csrc/schedule.cuh):
// runs the kernel's own planner and work iterator for every cluster of a
// grid and verifies what the kernel relies on.
//
//   schedule_check                    sweep of tile counts, parts, clusters
//   schedule_check T Q C SPLIT        one case, units printed
//
// Per case:
//   1. every column part of every tile is computed by exactly one unit;
//   2. units stay inside their tile (0 <= q0, q0 + w <= Q, w >= 1);
//   3. whole tiles come first and fill complete waves (dp_tiles % C == 0
//      whenever anything is split), and a cluster's units are whole tiles
//      first, then at most two runs of parts;
//   4. no cluster computes more parts of split tiles than the plan's run;
//   5. the grid covers every cluster that has work, within the resident ones;
//   6. done() is true exactly when next() has nothing left.
// Exit status 0 when every case holds.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "schedule.cuh"

namespace {

struct Params {
  int dp_tiles, tail_parts, tail_clusters;
};

int g_fail = 0;

void fail(const char* what, int t, int q, int c, int split) {
  if (g_fail < 20) std::printf("FAIL %s (tiles=%d parts=%d clusters=%d split=%d)\n", what, t, q, c, split);
  ++g_fail;
}

template <int Q>
bool check_case(int tiles, int clusters, int split, bool print) {
  const bm::Plan pl = bm::plan_schedule(tiles, Q, clusters, split);
  const Params p{pl.dp_tiles, pl.tail_parts, pl.tail_clusters};
  const int before = g_fail;
  const bool splits = pl.tail_parts > 0;
  if (splits && pl.dp_tiles % clusters != 0) fail("whole tiles not full waves", tiles, Q, clusters, split);
  if (splits && pl.tail_parts != (tiles - pl.dp_tiles) * Q) fail("tail part count", tiles, Q, clusters, split);
  if (pl.grid_clusters > clusters || pl.tail_clusters > pl.grid_clusters)
    fail("grid", tiles, Q, clusters, split);
  if (!split && splits) fail("split while disabled", tiles, Q, clusters, split);
  const int run = splits ? (pl.tail_parts + clusters - 1) / clusters : Q;
  std::vector<int> cover(static_cast<size_t>(tiles) * Q, 0);
  for (int c = 0; c < pl.grid_clusters; ++c) {
    bm::WorkIter<Q> it(p, c, pl.grid_clusters);
    bm::WorkUnit u;
    int tail_q = 0, tail_units = 0;
    bool in_tail = false;
    while (true) {
      const bool done = it.done(p);
      const bool got = it.next(p, u);
      if (done == got) fail("done() disagrees with next()", tiles, Q, clusters, split);
      if (!got) break;
      if (print) std::printf("cluster %d: tile %d parts [%d,%d)\n", c, u.tile, u.q0, u.q0 + u.w);
      if (u.tile < 0 || u.tile >= tiles || u.w < 1 || u.q0 < 0 || u.q0 + u.w > Q) {
        fail("unit out of range", tiles, Q, clusters, split);
        continue;
      }
      const bool tail = u.tile >= pl.dp_tiles;
      if (!tail && (u.q0 != 0 || u.w != Q)) fail("whole tile not whole", tiles, Q, clusters, split);
      if (in_tail && !tail) fail("whole tile after split units", tiles, Q, clusters, split);
      in_tail = in_tail || tail;
      if (tail) {
        tail_q += u.w;
        ++tail_units;
      }
      for (int q = u.q0; q < u.q0 + u.w; ++q) cover[static_cast<size_t>(u.tile) * Q + q] += 1;
    }
    if (tail_q > run) fail("cluster exceeds its run", tiles, Q, clusters, split);
    if (tail_units > 2) fail("more than two split units", tiles, Q, clusters, split);
  }
  for (size_t i = 0; i < cover.size(); ++i)
    if (cover[i] != 1) {
      fail("part not covered exactly once", tiles, Q, clusters, split);
      break;
    }
  return g_fail == before;
}

template <int Q>
long long sweep() {
  long long n = 0;
  for (int clusters : {1, 2, 3, 7, 16, 37, 64, 74, 148})
    for (int tiles = 1; tiles <= 4 * clusters + 3; ++tiles)
      for (int split = 0; split <= 1; ++split) {
        check_case<Q>(tiles, clusters, split, false);
        ++n;
      }
  return n;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc == 5) {
    const int t = std::atoi(argv[1]), q = std::atoi(argv[2]), c = std::atoi(argv[3]), s = std::atoi(argv[4]);
    bool ok = false;
    switch (q) {
      case 1: ok = check_case<1>(t, c, s, true); break;
      case 2: ok = check_case<2>(t, c, s, true); break;
      case 4: ok = check_case<4>(t, c, s, true); break;
      default: std::printf("parts must be 1, 2 or 4\n"); return 2;
    }
    const bm::Plan pl = bm::plan_schedule(t, q, c, s);
    std::printf("plan dp_tiles=%d tail_parts=%d tail_clusters=%d grid=%d est=%.4f\n", pl.dp_tiles,
                pl.tail_parts, pl.tail_clusters, pl.grid_clusters, pl.est);
    return ok ? 0 : 1;
  }
  const long long n = sweep<1>() + sweep<2>() + sweep<4>();
  std::printf("%lld cases, %d failures\n", n, g_fail);
  return g_fail == 0 ? 0 : 1;
}
