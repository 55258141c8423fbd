// Benchmark entry: parse -> check problem and device -> prepare the selected
// backend -> validate, warm up, time, validate -> print key=value results.
// Same command line and output keys as the reference's benchmark_host.cu; the
// backend is chosen at compile time with -DGEMM_KERNEL_HEADER="..." and the
// device gate admits compute capability 10.0 (B200, sm_100a).
#include "../host/driver.hpp"

#ifndef GEMM_KERNEL_HEADER
#define GEMM_KERNEL_HEADER "../kernels/sm100_fp16_gemm.cuh"
#endif
#include GEMM_KERNEL_HEADER

static_assert(gemm_backend::kInterfaceVersion == 1, "Unsupported GEMM backend interface");

static gemm_bench::BenchResult run_benchmark(const gemm_bench::BenchmarkOptions& options) {
  using namespace gemm_bench;
  GemmBuffers buffers(options);  // inputs built and copied before any timing
  auto validate = [&](const char* phase) {
    validate_gemm_output(phase, options.problem, buffers.h_A, buffers.h_B, buffers.h_C,
                         buffers.d_C);
  };
  auto measure = [&](const auto& launch, const LaunchConfig& config) {
    PerformanceStats stats =
        measure_gemm_performance(launch, validate, options.problem, options.measurement);
    return BenchResult{stats, config};
  };
  return gemm_backend::with_prepared(options, buffers, measure);
}

int main(int argc, char** argv) {
  using namespace gemm_bench;
  if (argc == 2 && (std::strcmp(argv[1], "--help") == 0 || std::strcmp(argv[1], "-h") == 0)) {
    std::cout << "Kernel: " << gemm_backend::kName << "\nKernel header: " << GEMM_KERNEL_HEADER
              << '\n';
    gemm_backend::print_configuration();
    print_usage(argv[0]);
    return EXIT_SUCCESS;
  }
  BenchmarkOptions options = parse_options(argc, argv);
  validate_options(options);
  gemm_backend::validate_problem(options.problem);

  cudaDeviceProp props{};
  int device = 0;
  BM_CUDA_CHECK(cudaGetDevice(&device));
  BM_CUDA_CHECK(cudaGetDeviceProperties(&props, device));
  if (props.major != 10 || props.minor != 0) {
    std::cerr << "This benchmark requires B200 / compute capability 10.0; device " << props.name
              << " has compute capability " << props.major << '.' << props.minor << '\n';
    return EXIT_FAILURE;
  }
  std::cout << "Kernel: " << gemm_backend::kName << "\nKernel header: " << GEMM_KERNEL_HEADER
            << '\n';
  print_configuration(props, options);
  gemm_backend::print_configuration();
  BenchResult result = run_benchmark(options);
  print_result(options, result);
  return EXIT_SUCCESS;
}
