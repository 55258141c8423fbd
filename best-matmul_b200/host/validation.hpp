// Output validation of the benchmark harness (outside any timed region).
//
// As in the reference (host/validation.cuh): copy all of C back, reject
// NaN/Inf, print a checksum, and compare a 4 x 4 grid of entries (corners
// included) against an FP64 dot product of the FP16 inputs with the
// reference's empirical tolerance 1 + 2 % |ref|. In addition every sampled
// entry (the grid plus 48 fixed pseudo-random ones) must meet the BASELINE
// per-element tolerance |c - ref| <= 1e-2 |ref| + 2e-3 sqrt(K / 4096).
#pragma once

#include <cmath>

#include "common.hpp"

namespace gemm_bench {

inline double copy_output_and_checksum(std::vector<Element>& out, const DeviceArray<Element>& d) {
  d.download(out);
  double sum = 0.0;
  for (std::size_t i = 0; i < out.size(); ++i) {
    const double v = static_cast<double>(__half2float(out[i]));
    if (!std::isfinite(v)) {
      std::cerr << "Non-finite GEMM output at " << i << '\n';
      std::exit(EXIT_FAILURE);
    }
    sum += v;
  }
  return sum;
}

// C(row, col) in FP64 from the FP16 inputs, in k order.
inline double reference_gemm_entry(const GemmProblem& p, const std::vector<Element>& A,
                                   const std::vector<Element>& B, int row, int col) {
  double acc = 0.0;
  for (int q = 0; q < p.k; ++q) {
    acc += static_cast<double>(__half2float(A[p.a_index(row, q)])) *
           static_cast<double>(__half2float(B[p.b_index(col, q)]));
  }
  return acc;
}

inline void validate_gemm_output(const char* phase, const GemmProblem& p,
                                 const std::vector<Element>& A, const std::vector<Element>& B,
                                 std::vector<Element>& C, const DeviceArray<Element>& d_C) {
  using namespace benchmark_policy;
  const double checksum = copy_output_and_checksum(C, d_C);
  double max_err = 0.0;
  constexpr int kAxis = kValidationAxisSamples;
  std::vector<std::pair<int, int>> samples;
  for (int r = 0; r < kAxis; ++r)
    for (int c = 0; c < kAxis; ++c)
      samples.emplace_back(static_cast<int>(static_cast<long long>(p.m - 1) * r / (kAxis - 1)),
                           static_cast<int>(static_cast<long long>(p.n - 1) * c / (kAxis - 1)));
  const std::size_t grid = samples.size();
  uint64_t h = 0x2545F4914F6CDD1Dull;  // fixed xorshift stream for the extra samples
  for (int i = 0; i < 48; ++i) {
    h ^= h << 13; h ^= h >> 7; h ^= h << 17;
    samples.emplace_back(static_cast<int>(h % static_cast<uint64_t>(p.m)),
                         static_cast<int>((h >> 32) % static_cast<uint64_t>(p.n)));
  }
  const double strict_abs = kStrictAbsTolerance * std::sqrt(p.k / 4096.0);
  double strict_max = 0.0;
  for (std::size_t s = 0; s < samples.size(); ++s) {
    const int row = samples[s].first, col = samples[s].second;
    const double ref = reference_gemm_entry(p, A, B, row, col);
    const double got = static_cast<double>(__half2float(C[p.c_index(row, col)]));
    const double err = std::abs(got - ref);
    if (s < grid) {
      max_err = std::max(max_err, err);
      if (err > kValidationAbsTolerance + kValidationRelativeTolerance * std::abs(ref)) {
        std::cerr << "Sampled GEMM validation failed at (" << row << ',' << col
                  << "): actual=" << got << ", reference=" << ref << '\n';
        std::exit(EXIT_FAILURE);
      }
    }
    strict_max = std::max(strict_max, err);
    if (err > kStrictRelativeTolerance * std::abs(ref) + strict_abs) {
      std::cerr << "Strict GEMM validation failed at (" << row << ',' << col
                << "): actual=" << got << ", reference=" << ref << '\n';
      std::exit(EXIT_FAILURE);
    }
  }
  std::cout << "Validation [" << phase << "]: " << grid << " sampled entries PASS, max_abs_error="
            << max_err << ", checksum=" << checksum << std::endl;
  std::cout << "Strict validation [" << phase << "]: " << samples.size()
            << " entries within 1e-2*|ref|+2e-3*sqrt(K/4096), max_abs_error=" << strict_max
            << std::endl;
}

}  // namespace gemm_bench
