// Problem, input and launch types of the benchmark harness.
//
// Same data contract as the reference harness (host/common.cuh): FP16 inputs
// and output, C = A * B^T with alpha = 1, beta = 0, logical shapes A(M,K),
// B(N,K), C(M,N), NT/TN physical layouts and column-major C. Input modes 0..3
// reproduce the reference's values exactly (same std::rand() sequence for mode
// 2); modes 4 and 5 add the BASELINE distributions. Device memory is plain
// cudaMalloc owned by RAII holders (the reference uses thrust vectors).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <utility>
#include <vector>

#include "../csrc/bm_inputs.cuh"

// Abort-with-message on CUDA errors: the harness must never record numbers
// from a failed run (reference: CUTE_CHECK_ERROR + std::exit, benchmark_host.cu:68).
#define BM_CUDA_CHECK(expr)                                                              \
  do {                                                                                   \
    cudaError_t bm_err_ = (expr);                                                        \
    if (bm_err_ != cudaSuccess) {                                                        \
      std::fprintf(stderr, "CUDA error %s at %s:%d: %s\n", cudaGetErrorName(bm_err_),    \
                   __FILE__, __LINE__, cudaGetErrorString(bm_err_));                    \
      std::exit(EXIT_FAILURE);                                                           \
    }                                                                                    \
  } while (0)

namespace gemm_bench {

using Element = __half;

enum class InputMode {
  Zero = 0,       // C = 0: catches missing writes when C is NaN-prefilled
  One = 1,        // C = K everywhere
  RandomPm1 = 2,  // +-1 from std::rand() after srand(0): the reference default
  Pattern = 3,    // ((physical index + 17 * matrix) % 5) - 2
  Uniform = 4,    // uniform[-1, 1), counter-based, seed 0
  Normal = 5,     // ~N(0, 0.02), counter-based, seed 0
};

enum class TimerMode { Wall, Event };

inline const char* timer_mode_name(TimerMode m) { return m == TimerMode::Event ? "event" : "wall"; }

// Logical A(M,K), B(N,K), C(M,N); C(m,n) = sum_k A(m,k) * B(n,k).
// NT: M / N contiguous in A / B; TN: K contiguous; C column-major.
struct GemmProblem {
  int m = 4096;
  int n = 4096;
  int k = 4096;
  char transA = 'N';
  char transB = 'T';

  bool is_nt() const { return transA == 'N' && transB == 'T'; }
  int ldA() const { return transA == 'N' ? m : k; }
  int ldB() const { return transB == 'T' ? n : k; }
  int ldC() const { return m; }
  std::size_t a_elements() const { return std::size_t(m) * std::size_t(k); }
  std::size_t b_elements() const { return std::size_t(n) * std::size_t(k); }
  std::size_t c_elements() const { return std::size_t(m) * std::size_t(n); }
  std::size_t a_index(int row, int p) const {
    return transA == 'N' ? std::size_t(row) + std::size_t(p) * std::size_t(ldA())
                         : std::size_t(row) * std::size_t(ldA()) + std::size_t(p);
  }
  std::size_t b_index(int col, int p) const {
    return transB == 'T' ? std::size_t(col) + std::size_t(p) * std::size_t(ldB())
                         : std::size_t(col) * std::size_t(ldB()) + std::size_t(p);
  }
  std::size_t c_index(int row, int col) const {
    return std::size_t(row) + std::size_t(col) * std::size_t(ldC());
  }
};

struct MeasurementConfig {
  TimerMode timer_mode = TimerMode::Event;
  int launches_per_batch = 20;
  int min_warmup_launches = 20;
  int batches = 200;
  cudaStream_t stream = nullptr;
};

struct BenchmarkOptions {
  GemmProblem problem;
  InputMode input_mode = InputMode::RandomPm1;
  MeasurementConfig measurement;
};

struct LaunchConfig {
  int smem_bytes = 0;
  dim3 grid{1, 1, 1};
  dim3 block{1, 1, 1};
  dim3 cluster{1, 1, 1};
};

// Empirical thresholds of the measurement and validation policy (the
// reference's benchmark_policy values, host/common.cuh:100-109).
namespace benchmark_policy {
constexpr std::size_t kWarmupWindowBatches = 5;
constexpr int kStableWindowCount = 2;
constexpr int kExtraWarmupBatches = 20;
constexpr double kPlateauRelativeTolerance = 0.02;
constexpr double kDriftWarningPct = 5.0;
constexpr int kValidationAxisSamples = 4;
constexpr double kValidationAbsTolerance = 1.0;
constexpr double kValidationRelativeTolerance = 0.02;
// BASELINE per-element tolerance: |c - ref| <= 1e-2 |ref| + 2e-3 sqrt(K / 4096)
constexpr double kStrictRelativeTolerance = 1e-2;
constexpr double kStrictAbsTolerance = 2e-3;
}  // namespace benchmark_policy

// One input value. `physical` is the element's index in its buffer (modes 2
// and 3 depend on it, as in the reference); `logical` is row * K + k of the
// logical matrix (modes 4 and 5, so any row block regenerates identically).
inline Element make_input_value(std::size_t physical, std::size_t logical, int matrix_id,
                                InputMode mode) {
  switch (mode) {
    case InputMode::Zero: return __float2half(0.0f);
    case InputMode::One: return __float2half(1.0f);
    case InputMode::RandomPm1: return __float2half(std::rand() % 2 ? 1.0f : -1.0f);
    case InputMode::Pattern:
    case InputMode::Uniform:
    case InputMode::Normal: {
      const uint64_t key = bm::input_key(0, matrix_id);
      return __float2half_rn(
          bm::input_value_f32(static_cast<int>(mode), key, logical, physical, matrix_id));
    }
  }
  return __float2half(0.0f);
}

// Device buffer owned for the lifetime of the holder.
template <class T>
class DeviceArray {
 public:
  DeviceArray() = default;
  explicit DeviceArray(std::size_t n) : n_(n) {
    BM_CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&p_), n * sizeof(T)));
  }
  ~DeviceArray() {
    if (p_) cudaFree(p_);
  }
  DeviceArray(const DeviceArray&) = delete;
  DeviceArray& operator=(const DeviceArray&) = delete;
  DeviceArray(DeviceArray&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr; o.n_ = 0; }
  DeviceArray& operator=(DeviceArray&& o) noexcept {
    std::swap(p_, o.p_);
    std::swap(n_, o.n_);
    return *this;
  }
  T* get() const { return p_; }
  std::size_t size() const { return n_; }
  void upload(const std::vector<T>& h) {
    BM_CUDA_CHECK(cudaMemcpy(p_, h.data(), n_ * sizeof(T), cudaMemcpyHostToDevice));
  }
  void download(std::vector<T>& h) const {
    h.resize(n_);
    BM_CUDA_CHECK(cudaMemcpy(h.data(), p_, n_ * sizeof(T), cudaMemcpyDeviceToHost));
  }

 private:
  T* p_ = nullptr;
  std::size_t n_ = 0;
};

// Host inputs in physical order, their device copies, and C (zeroed).
// Generation and host->device copies happen before any timing.
struct GemmBuffers {
  std::vector<Element> h_A, h_B, h_C;
  DeviceArray<Element> d_A, d_B, d_C;

  explicit GemmBuffers(const BenchmarkOptions& options)
      : h_A(options.problem.a_elements()),
        h_B(options.problem.b_elements()),
        h_C(options.problem.c_elements(), __float2half(0.0f)),
        d_A(options.problem.a_elements()),
        d_B(options.problem.b_elements()),
        d_C(options.problem.c_elements()) {
    const GemmProblem& p = options.problem;
    std::srand(0);  // one fixed sequence shared by A then B (mode 2)
    for (std::size_t i = 0; i < h_A.size(); ++i) {
      const std::size_t row = p.is_nt() ? i % p.m : i / p.k;
      const std::size_t col = p.is_nt() ? i / p.m : i % p.k;
      h_A[i] = make_input_value(i, row * p.k + col, 0, options.input_mode);
    }
    for (std::size_t i = 0; i < h_B.size(); ++i) {
      const std::size_t row = p.is_nt() ? i % p.n : i / p.k;
      const std::size_t col = p.is_nt() ? i / p.n : i % p.k;
      h_B[i] = make_input_value(i, row * p.k + col, 1, options.input_mode);
    }
    d_A.upload(h_A);
    d_B.upload(h_B);
    d_C.upload(h_C);
  }
};

}  // namespace gemm_bench
