// Timing, warm-up and statistics of the benchmark harness.
//
// Contract kept from the reference harness (host/measurement.cuh):
//  - a sample is the average per-launch time of one batch of back-to-back
//    launches on one stream (CUDA events, or a steady clock + stream sync);
//  - warm-up runs until the median of the last 5-batch window is within 2 %
//    of the previous window twice in a row (at least min_warmup launches,
//    at most 20 extra batches), and reports whether the plateau was reached;
//  - p50/p99 use linear interpolation between order statistics; drift is the
//    last-quarter median over the first-quarter median;
//  - TFLOP/s = 2 M N K / latency;
//  - validation runs before warm-up and after sampling, never inside timing.
// The launch callback only enqueues work on config.stream.
#pragma once

#include <algorithm>
#include <chrono>
#include <cmath>
#include <limits>
#include <numeric>
#include <vector>

#include "common.hpp"

namespace gemm_bench {

struct PerformanceStats {
  std::size_t sample_count = 0;
  double elapsed_ms = 0.0;
  double p50_ms = 0.0;
  double p99_ms = 0.0;
  double min_ms = 0.0;
  double max_ms = 0.0;
  double drift_pct = 0.0;
  double tflops_p50 = 0.0;
  double tflops_at_p99_latency = 0.0;
  int warmup_launches = 0;
  bool warmup_stable = false;
};

inline void validate_measurement_config(const MeasurementConfig& c) {
  if (c.min_warmup_launches <= 0 || c.launches_per_batch <= 0 || c.batches < 2) {
    std::cerr << "Require min_warmup > 0, per_batch > 0, batches >= 2\n";
    std::exit(EXIT_FAILURE);
  }
  const long long worst = static_cast<long long>(c.min_warmup_launches) +
                          (benchmark_policy::kExtraWarmupBatches + 1LL) * c.launches_per_batch;
  if (worst > std::numeric_limits<int>::max()) {
    std::cerr << "Warmup count exceeds supported integer range\n";
    std::exit(EXIT_FAILURE);
  }
}

// Times batches of launches; owns its two events.
class BatchTimer {
 public:
  explicit BatchTimer(const MeasurementConfig& c) : mode_(c.timer_mode), stream_(c.stream) {
    if (mode_ == TimerMode::Event) {
      BM_CUDA_CHECK(cudaEventCreate(&t0_));
      BM_CUDA_CHECK(cudaEventCreate(&t1_));
    }
  }
  ~BatchTimer() {
    if (mode_ == TimerMode::Event) {
      cudaEventDestroy(t0_);
      cudaEventDestroy(t1_);
    }
  }
  BatchTimer(const BatchTimer&) = delete;
  BatchTimer& operator=(const BatchTimer&) = delete;

  // Average per-launch milliseconds of `count` back-to-back launches.
  template <class Launch>
  double measure(const Launch& launch, int count) {
    std::chrono::steady_clock::time_point h0;
    if (mode_ == TimerMode::Event) BM_CUDA_CHECK(cudaEventRecord(t0_, stream_));
    else h0 = std::chrono::steady_clock::now();
    for (int i = 0; i < count; ++i) launch();
    BM_CUDA_CHECK(cudaGetLastError());
    double ms;
    if (mode_ == TimerMode::Event) {
      BM_CUDA_CHECK(cudaEventRecord(t1_, stream_));
      BM_CUDA_CHECK(cudaEventSynchronize(t1_));
      float f = 0.0f;
      BM_CUDA_CHECK(cudaEventElapsedTime(&f, t0_, t1_));
      ms = f;
    } else {
      BM_CUDA_CHECK(cudaStreamSynchronize(stream_));
      ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - h0).count();
    }
    if (!std::isfinite(ms) || ms <= 0.0) {
      std::cerr << "Timer resolution insufficient; increase per_batch\n";
      std::exit(EXIT_FAILURE);
    }
    return ms / count;
  }

 private:
  TimerMode mode_;
  cudaStream_t stream_;
  cudaEvent_t t0_{}, t1_{};
};

// q-quantile of ascending samples, linear between neighbours (q*(n-1)).
inline double quantile_sorted(const std::vector<double>& s, double q) {
  if (s.empty() || !(q >= 0.0 && q <= 1.0)) {
    std::cerr << "Invalid percentile input\n";
    std::exit(EXIT_FAILURE);
  }
  const double pos = q * static_cast<double>(s.size() - 1);
  const std::size_t lo = static_cast<std::size_t>(pos);
  const std::size_t hi = std::min(lo + 1, s.size() - 1);
  return s[lo] + (pos - static_cast<double>(lo)) * (s[hi] - s[lo]);
}

inline double median_of(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  return quantile_sorted(v, 0.5);
}

inline double window_median(const std::vector<double>& v, std::size_t first, std::size_t n) {
  return median_of(std::vector<double>(v.begin() + first, v.begin() + first + n));
}

struct WarmupResult {
  int launches = 0;
  bool stable = false;
};

template <class Launch>
WarmupResult warmup_until_stable(BatchTimer& timer, const Launch& launch, const MeasurementConfig& c) {
  using namespace benchmark_policy;
  const int needed = static_cast<int>((static_cast<long long>(c.min_warmup_launches) +
                                       c.launches_per_batch - 1) / c.launches_per_batch);
  const int limit = needed + kExtraWarmupBatches;
  std::vector<double> samples;
  WarmupResult r;
  int calm = 0;
  for (int b = 0; b < limit; ++b) {
    samples.push_back(timer.measure(launch, c.launches_per_batch));
    r.launches += c.launches_per_batch;
    const std::size_t n = samples.size();
    if (n < 2 * kWarmupWindowBatches || n % kWarmupWindowBatches != 0) continue;
    const double before = window_median(samples, n - 2 * kWarmupWindowBatches, kWarmupWindowBatches);
    const double now = window_median(samples, n - kWarmupWindowBatches, kWarmupWindowBatches);
    calm = (std::abs(now / before - 1.0) <= kPlateauRelativeTolerance) ? calm + 1 : 0;
    if (static_cast<int>(n) >= needed && calm >= kStableWindowCount) {
      r.stable = true;
      break;
    }
  }
  return r;
}

inline double gemm_tflops(const GemmProblem& p, double ms) {
  if (p.m <= 0 || p.n <= 0 || p.k <= 0 || !std::isfinite(ms) || ms <= 0.0) {
    std::cerr << "Invalid GEMM dimensions or latency\n";
    std::exit(EXIT_FAILURE);
  }
  return 2.0 * double(p.m) * double(p.n) * double(p.k) / (ms * 1.0e9);
}

inline PerformanceStats summarize_performance(const std::vector<double>& samples, int per_batch,
                                              const GemmProblem& p) {
  if (samples.size() < 2 || per_batch <= 0) {
    std::cerr << "Need at least two batches and positive launches per batch\n";
    std::exit(EXIT_FAILURE);
  }
  for (double s : samples) {
    if (!std::isfinite(s) || s <= 0.0) {
      std::cerr << "Invalid elapsed time; increase launches per batch\n";
      std::exit(EXIT_FAILURE);
    }
  }
  std::vector<double> sorted = samples;
  std::sort(sorted.begin(), sorted.end());
  PerformanceStats st;
  st.sample_count = samples.size();
  st.elapsed_ms = std::accumulate(samples.begin(), samples.end(), 0.0) * per_batch;
  st.p50_ms = quantile_sorted(sorted, 0.5);
  st.p99_ms = quantile_sorted(sorted, 0.99);
  st.min_ms = sorted.front();
  st.max_ms = sorted.back();
  st.tflops_p50 = gemm_tflops(p, st.p50_ms);
  st.tflops_at_p99_latency = gemm_tflops(p, st.p99_ms);
  const std::size_t w = std::max<std::size_t>(1, samples.size() / 4);
  st.drift_pct = 100.0 * (window_median(samples, samples.size() - w, w) /
                          window_median(samples, 0, w) - 1.0);
  return st;
}

// GPU state snapshot via nvidia-smi, outside the timed region; selected by
// PCI bus id so CUDA_VISIBLE_DEVICES remapping cannot pick the wrong GPU.
inline void print_gpu_state(const char* phase) {
  int dev = 0;
  char bus[32] = {};
  BM_CUDA_CHECK(cudaGetDevice(&dev));
  BM_CUDA_CHECK(cudaDeviceGetPCIBusId(bus, sizeof(bus), dev));
  std::cout << "GPU state [" << phase << "] PCI=" << bus << std::endl;
  char cmd[512];
  std::snprintf(cmd, sizeof(cmd),
                "nvidia-smi -i %s --query-gpu=timestamp,uuid,driver_version,pstate,"
                "temperature.gpu,power.draw,clocks.sm,clocks.mem,utilization.gpu,memory.used "
                "--format=csv",
                bus);
  std::fflush(stdout);
  if (std::system(cmd) != 0) std::cout << "GPU telemetry unavailable (nvidia-smi); measurement continues\n";
}

// precheck -> warm-up -> sampled batches -> postcheck -> summary.
template <class Launch, class Validate>
PerformanceStats measure_gemm_performance(const Launch& launch, const Validate& validate,
                                          const GemmProblem& problem, const MeasurementConfig& c) {
  validate_measurement_config(c);
  BatchTimer timer(c);
  print_gpu_state("start");
  launch();
  BM_CUDA_CHECK(cudaGetLastError());
  BM_CUDA_CHECK(cudaStreamSynchronize(c.stream));
  validate("precheck");
  const WarmupResult wu = warmup_until_stable(timer, launch, c);
  if (!wu.stable) std::cerr << "Warning: warmup did not reach a stable plateau; interpret results cautiously\n";
  std::cout << "Warmup launches=" << wu.launches
            << ", plateau=" << (wu.stable ? "stable" : "not confirmed") << std::endl;
  std::vector<double> samples;
  samples.reserve(static_cast<std::size_t>(c.batches));
  for (int b = 0; b < c.batches; ++b) samples.push_back(timer.measure(launch, c.launches_per_batch));
  print_gpu_state("end");
  validate("postcheck");
  PerformanceStats st = summarize_performance(samples, c.launches_per_batch, problem);
  st.warmup_launches = wu.launches;
  st.warmup_stable = wu.stable;
  return st;
}

}  // namespace gemm_bench
