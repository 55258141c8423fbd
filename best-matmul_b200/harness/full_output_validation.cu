// Full-output regression for the selected backend (the pattern of the
// reference's tests/full_output_validation.cu):
//  1. host-only: the epilogue's (warp, lane, chunk, step) -> C coordinate map
//     covers every element of a CTA's 128 x tile_n output exactly once;
//  2. on a B200: for NT and TN, input modes 0..3 and K-tile counts
//     {1, 2, S-1, S, S+1, 3S+1} (S = pipeline stages), M = 2 tile rows and
//     N = 2 tile columns, C prefilled with NaN, two launches, and every
//     element of C compared bit for bit with the FP16 rounding of the exact
//     integer result (FP32 accumulation of these integers is exact).
// Usage: full_output_validation [--mapping-only]
#include <set>

#include "../csrc/gemm_sm100.cuh"
#include "../host/driver.hpp"

#ifndef GEMM_KERNEL_HEADER
#define GEMM_KERNEL_HEADER "../kernels/sm100_fp16_gemm.cuh"
#endif
#include GEMM_KERNEL_HEADER

namespace {

struct Geometry {
  int variant, tile_m, tile_n, stages;
};

// Geometry of the backend's variant for a representative problem.
Geometry backend_geometry() {
  static const int tiles[6][3] = {{0, 0, 0}, {256, 256, 6}, {128, 256, 4},
                                  {128, 128, 6}, {256, 128, 6}, {256, 512, 4}};
  int v = gemm_backend::kVariant;
  if (v == 0) v = BM_VARIANT_2CTA_256x512;  // what auto picks for large squares
  return Geometry{v, tiles[v][0], tiles[v][1], tiles[v][2]};
}

bool check_output_mapping(int tile_n) {
  const int chunks = tile_n / 32, per_warp = chunks / 2;
  std::vector<int> owners(static_cast<std::size_t>(128) * tile_n, 0);
  for (int warp = 2; warp < 2 + bm::kEpiWarps; ++warp)
    for (int lane = 0; lane < 32; ++lane)
      for (int cc = 0; cc < per_warp; ++cc)
        for (int i = 0; i < 16; ++i) {
          const int c = bm::epi_chunk(warp, cc, per_warp, bm::epi_half_order(tile_n));
          // each lane stores one word = rows (row, row + 1) of one column
          const bm::EpiCoord e = bm::epi_word_coord(warp, lane, c, i);
          for (int r = 0; r < 2; ++r) {
            const int row = e.row + r;
            if (row < 0 || row >= 128 || e.col < 0 || e.col >= tile_n) {
              std::cerr << "Mapping out of bounds: warp " << warp << " lane " << lane << '\n';
              return false;
            }
            ++owners[static_cast<std::size_t>(row) + static_cast<std::size_t>(e.col) * 128];
          }
        }
  // each element is written by exactly one lane (the word of its row pair)
  for (std::size_t i = 0; i < owners.size(); ++i) {
    if (owners[i] != 1) {
      std::cerr << "Output ownership count=" << owners[i] << " at linear coordinate " << i << '\n';
      return false;
    }
  }
  // TMEM lane quarters: warp w may only read lanes 32*(w%4)..; two warps each
  for (int q = 0; q < 4; ++q) {
    int n = 0;
    for (int warp = 2; warp < 2 + bm::kEpiWarps; ++warp) n += bm::epi_quarter(warp) == q;
    if (n != 2) {
      std::cerr << "TMEM lane quarter " << q << " has " << n << " epilogue warps\n";
      return false;
    }
  }
  std::cout << "Mapping PASS: " << bm::kEpiWarps * 32 << " epilogue threads cover 128 x " << tile_n
            << " output coordinates exactly once\n";
  return true;
}

bool check_case(bool nt, int k_tiles, gemm_bench::InputMode input, const Geometry& g) {
  using namespace gemm_bench;
  BenchmarkOptions o;
  o.problem.m = 2 * g.tile_m;
  o.problem.n = 2 * g.tile_n;
  o.problem.k = k_tiles * 64;
  o.problem.transA = nt ? 'N' : 'T';
  o.problem.transB = nt ? 'T' : 'N';
  o.input_mode = input;
  gemm_backend::validate_problem(o.problem);
  GemmBuffers buf(o);
  std::vector<Element> nan_fill(o.problem.c_elements(), __float2half(NAN));
  buf.d_C.upload(nan_fill);
  return gemm_backend::with_prepared(o, buf, [&](const auto& launch, const LaunchConfig&) {
    launch();
    launch();  // stale pipeline state and beta = 0 overwrite
    BM_CUDA_CHECK(cudaGetLastError());
    BM_CUDA_CHECK(cudaStreamSynchronize(o.measurement.stream));
    buf.d_C.download(buf.h_C);
    const GemmProblem& p = o.problem;
    for (int col = 0; col < p.n; ++col) {
      for (int row = 0; row < p.m; ++row) {
        long long exact = 0;
        for (int q = 0; q < p.k; ++q)
          exact += static_cast<long long>(__half2float(buf.h_A[p.a_index(row, q)])) *
                   static_cast<long long>(__half2float(buf.h_B[p.b_index(col, q)]));
        const __half want = __float2half_rn(static_cast<float>(exact));
        const __half got = buf.h_C[p.c_index(row, col)];
        uint16_t wb, gb;
        std::memcpy(&wb, &want, 2);
        std::memcpy(&gb, &got, 2);
        if (wb != gb) {
          std::cerr << "Full-output failure: layout=" << (nt ? "NT" : "TN") << ", input="
                    << static_cast<int>(input) << ", K tiles=" << k_tiles << ", C(" << row << ','
                    << col << ")=" << __half2float(got) << ", reference=" << exact << '\n';
          return false;
        }
      }
    }
    std::cout << "Full-output PASS: " << (nt ? "NT" : "TN") << ", input=" << static_cast<int>(input)
              << ", K tiles=" << k_tiles << ", checked=" << p.c_elements() << '\n';
    return true;
  });
}

}  // namespace

int main(int argc, char** argv) {
  const bool mapping_only = argc == 2 && std::strcmp(argv[1], "--mapping-only") == 0;
  if (argc > 1 && !mapping_only) {
    std::cerr << "Usage: " << argv[0] << " [--mapping-only]\n";
    return EXIT_FAILURE;
  }
  const Geometry g = backend_geometry();
  std::cout << "Kernel: " << gemm_backend::kName << '\n';
  gemm_backend::print_configuration();
  if (!check_output_mapping(g.tile_n)) return EXIT_FAILURE;
  if (mapping_only) return EXIT_SUCCESS;
  cudaDeviceProp props{};
  int device = 0;
  BM_CUDA_CHECK(cudaGetDevice(&device));
  BM_CUDA_CHECK(cudaGetDeviceProperties(&props, device));
  if (props.major != 10 || props.minor != 0) {
    std::cerr << "Full-output validation requires B200 / compute capability 10.0; device "
              << props.name << " has " << props.major << '.' << props.minor
              << ". Use --mapping-only for host validation.\n";
    return EXIT_FAILURE;
  }
  std::set<int> tile_counts{1, 2, g.stages - 1, g.stages, g.stages + 1, 3 * g.stages + 1};
  tile_counts.erase(0);
  for (bool nt : {true, false})
    for (auto in : {gemm_bench::InputMode::Zero, gemm_bench::InputMode::One,
                    gemm_bench::InputMode::RandomPm1, gemm_bench::InputMode::Pattern})
      for (int t : tile_counts)
        if (!check_case(nt, t, in, g)) return EXIT_FAILURE;
  std::cout << "All full-output regressions PASS\n";
  return EXIT_SUCCESS;
}
