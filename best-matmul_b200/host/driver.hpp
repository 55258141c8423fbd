// Command line, option checks and result printing of the benchmark harness.
//
// The positional command line and the key=value result lines are the
// machine contract scripts parse (reference host/driver.cuh:18-26, 71-91,
// 131-158 and scripts/common/runner_common.sh:444-454), so names, order and
// defaults are kept: M N K transA transB input_mode event|wall per_batch
// min_warmup batches; p50_ms, p99_ms, TFLOPS_p50, warmup_launches,
// warmup_stable, batch_drift_pct. Input modes 4 (uniform[-1,1]) and 5
// (normal(0, 0.02)) are additions.
#pragma once

#include <cerrno>
#include <climits>
#include <cstring>
#include <iomanip>

#include "measurement.hpp"
#include "validation.hpp"

namespace gemm_bench {

struct BenchResult {
  PerformanceStats performance;
  LaunchConfig launch;
};

inline void print_usage(const char* program) {
  std::cout << "Usage: " << program
            << " [M N K transA transB input_mode event|wall per_batch min_warmup batches]\n"
            << "Defaults: 4096 4096 4096 N T 2 event 20 20 200\n"
            << "Modes: N T or T N; input_mode: 0=zero, 1=one, 2=random +/-1, 3=pattern, "
               "4=uniform[-1,1], 5=normal(0,0.02)\n"
            << "per_batch = launches per batch; min_warmup is a minimum, not a fixed count\n"
            << "p50/p99 describe batch-average per-launch latency\n";
}

[[noreturn]] inline void fail_option(const std::string& msg) {
  std::cerr << msg << '\n';
  std::exit(EXIT_FAILURE);
}

// Whole-string base-10 integer within int range ("20x", "" and overflow fail).
inline int parse_integer(const char* text, const char* name) {
  char* end = nullptr;
  errno = 0;
  const long v = std::strtol(text, &end, 10);
  if (errno == ERANGE || end == text || *end != '\0' || v < INT_MIN || v > INT_MAX)
    fail_option(std::string("Invalid integer for ") + name + ": " + text);
  return static_cast<int>(v);
}

inline char parse_transpose(const char* text, const char* name) {
  if (std::strlen(text) != 1) fail_option(std::string(name) + " must be one character");
  return text[0];
}

inline InputMode parse_input_mode(const char* text) {
  const int v = parse_integer(text, "input_mode");
  if (v < 0 || v > 5) fail_option("INPUT_MODE must be one of {0, 1, 2, 3, 4, 5}");
  return static_cast<InputMode>(v);
}

inline TimerMode parse_timer_mode(const char* text) {
  if (std::strcmp(text, "event") == 0) return TimerMode::Event;
  if (std::strcmp(text, "wall") == 0) return TimerMode::Wall;
  fail_option("Timer mode must be wall or event");
}

inline BenchmarkOptions parse_options(int argc, char** argv) {
  if (argc > 11) {
    print_usage(argv[0]);
    std::exit(EXIT_FAILURE);
  }
  BenchmarkOptions o;
  if (argc >= 2) o.problem.m = parse_integer(argv[1], "M");
  if (argc >= 3) o.problem.n = parse_integer(argv[2], "N");
  if (argc >= 4) o.problem.k = parse_integer(argv[3], "K");
  if (argc >= 5) o.problem.transA = parse_transpose(argv[4], "transA");
  if (argc >= 6) o.problem.transB = parse_transpose(argv[5], "transB");
  if (argc >= 7) o.input_mode = parse_input_mode(argv[6]);
  if (argc >= 8) o.measurement.timer_mode = parse_timer_mode(argv[7]);
  if (argc >= 9) o.measurement.launches_per_batch = parse_integer(argv[8], "per_batch");
  if (argc >= 10) o.measurement.min_warmup_launches = parse_integer(argv[9], "min_warmup");
  if (argc >= 11) o.measurement.batches = parse_integer(argv[10], "batches");
  return o;
}

inline void validate_options(const BenchmarkOptions& o) {
  const GemmProblem& p = o.problem;
  validate_measurement_config(o.measurement);
  if (p.m <= 0 || p.n <= 0 || p.k <= 0) fail_option("Require M,N,K > 0");
  const bool tn = p.transA == 'T' && p.transB == 'N';
  if (!p.is_nt() && !tn) fail_option("Only NT and TN modes are implemented. Use N T or T N");
  const std::size_t lim = static_cast<std::size_t>(INT_MAX);
  if (p.a_elements() > lim || p.b_elements() > lim || p.c_elements() > lim)
    fail_option("Matrix element count exceeds supported range");
}

inline void print_configuration(const cudaDeviceProp& props, const BenchmarkOptions& o) {
  const GemmProblem& p = o.problem;
  const MeasurementConfig& m = o.measurement;
  std::printf("Device: %s, SM count=%d, compute capability=%d.%d\n", props.name,
              props.multiProcessorCount, props.major, props.minor);
  std::printf("Input mode: INPUT_MODE=%d\n", static_cast<int>(o.input_mode));
  std::printf("MIN_WARMUP=%d, LAUNCHES_PER_BATCH=%d, BATCHES=%d\n", m.min_warmup_launches,
              m.launches_per_batch, m.batches);
  std::printf("Timer=%s, scope=%s\n", timer_mode_name(m.timer_mode),
              m.timer_mode == TimerMode::Event ? "GPU event interval"
                                               : "host submission + stream completion");
  std::printf("Problem: M=%d, N=%d, K=%d, mode=%c%c\n", p.m, p.n, p.k, p.transA, p.transB);
}

inline void print_result(const BenchmarkOptions& o, const BenchResult& r) {
  const GemmProblem& p = o.problem;
  const LaunchConfig& l = r.launch;
  const PerformanceStats& s = r.performance;
  std::cout << std::fixed << std::setprecision(6);
  std::cout << "Launch config: grid=(" << l.grid.x << ',' << l.grid.y << ',' << l.grid.z << ')'
            << ", block=" << l.block.x << ", cluster=(" << l.cluster.x << ',' << l.cluster.y << ','
            << l.cluster.z << ')' << ", smem=" << l.smem_bytes << " bytes\n"
            << "M=" << p.m << ", N=" << p.n << ", K=" << p.k << "\n"
            << "sample_scope=batch-average per-launch latency\n"
            << "n_batches=" << s.sample_count
            << ", launches_per_batch=" << o.measurement.launches_per_batch << "\n"
            << "warmup_launches=" << s.warmup_launches
            << ", warmup_stable=" << (s.warmup_stable ? "yes" : "no") << "\n"
            << "elapsed_ms_measured_batches=" << s.elapsed_ms << " ms\n"
            << "p50_ms=" << s.p50_ms << " ms\n"
            << "p99_ms=" << s.p99_ms << " ms\n"
            << "min_ms=" << s.min_ms << " ms\n"
            << "max_ms=" << s.max_ms << " ms\n"
            << "TFLOPS_p50=" << s.tflops_p50 << "\n"
            << "TFLOPS_at_p99_latency=" << s.tflops_at_p99_latency << "\n"
            << "batch_drift_pct=" << s.drift_pct << " % (last/first quarter medians)\n";
  if (std::abs(s.drift_pct) > benchmark_policy::kDriftWarningPct)
    std::cerr << "Warning: latency drift exceeds 5%; inspect GPU state and repeat the run\n";
}

}  // namespace gemm_bench
