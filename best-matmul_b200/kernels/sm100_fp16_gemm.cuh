// gemm_backend for the B200 (sm_100a) tcgen05 GEMM: the compile-time plugin
// selected with -DGEMM_KERNEL_HEADER, exposing the names the reference's
// harness binds (README.md:278-287, benchmark_host.cu:5-10,
// kernels/detail/tma_wgmma_adapter.cuh:134-168):
//
//   gemm_backend::kInterfaceVersion, kName, validate_problem(),
//   print_configuration(), with_prepared(options, buffers, runner)
//
// It is a thin C++ layer over the C ABI in include/bm_gemm.h: with_prepared()
// calls bm_gemm_prepare once, hands the runner a zero-argument launch() that
// only enqueues bm_gemm_launch on the measurement stream, checks the kernel's
// status word after the runner returns and destroys the handle. Failures exit
// non-zero, like the reference, so scripts never record numbers from a failed
// configuration.
//
// Like every GEMM_KERNEL_HEADER, it is included after the harness has declared
// gemm_bench::GemmProblem, BenchmarkOptions, GemmBuffers and LaunchConfig; it
// uses only their member names, so it compiles against this repository's
// harness (host/*.hpp) and against the reference's (host/*.cuh, whose
// GemmBuffers hold thrust::device_vector).
//
// Compile-time knobs (recorded in manifest.tsv by build.sh):
//   SM100_VARIANT  0 = choose from the shape, 1..5 = a fixed bm_variant
//   SM100_STRICT   1 = reject shapes that are not tile multiples (the
//                  reference's validate_problem); 0 = accept ragged shapes
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <type_traits>
#include <utility>

#include "../../include/bm_gemm.h"

#ifndef SM100_VARIANT
#define SM100_VARIANT 0
#endif
#ifndef SM100_STRICT
#define SM100_STRICT 1
#endif

namespace gemm_backend {

constexpr int kInterfaceVersion = 1;
constexpr int kVariant = SM100_VARIANT;
constexpr bool kStrictTiles = SM100_STRICT != 0;
#if SM100_VARIANT == 1
constexpr char kName[] = "sm100_tcgen05_2cta_256x256x64_s6";
#elif SM100_VARIANT == 2
constexpr char kName[] = "sm100_tcgen05_1cta_128x256x64_s4";
#elif SM100_VARIANT == 3
constexpr char kName[] = "sm100_tcgen05_1cta_128x128x64_s6";
#elif SM100_VARIANT == 4
constexpr char kName[] = "sm100_tcgen05_2cta_256x128x64_s6";
#elif SM100_VARIANT == 5
constexpr char kName[] = "sm100_tcgen05_2cta_256x512x64_s4";
#else
constexpr char kName[] = "sm100_tcgen05_auto";
#endif

namespace detail {

// Device address held by a harness buffer: thrust::device_vector exposes
// data().get(), this repository's DeviceArray exposes get().
template <class V, class = void>
struct has_thrust_data : std::false_type {};
template <class V>
struct has_thrust_data<V, std::void_t<decltype(std::declval<V&>().data().get())>> : std::true_type {};

template <class V>
void* device_pointer(V& v) {
  if constexpr (has_thrust_data<V>::value) {
    return static_cast<void*>(v.data().get());
  } else {
    return static_cast<void*>(v.get());
  }
}

template <class Problem>
bm_gemm_desc make_desc(const Problem& p, const void* a, const void* b, void* c) {
  bm_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.m = p.m;
  d.n = p.n;
  d.k = p.k;
  d.trans_a = p.transA;
  d.trans_b = p.transB;
  d.a = a;
  d.b = b;
  d.c = c;
  d.variant = kVariant;
  d.strict_tiles = kStrictTiles ? 1 : 0;
  return d;
}

[[noreturn]] inline void die(const char* what, int code) {
  std::cerr << "Error: " << what << ": " << bm_gemm_error_string(code) << " (" << code << ")\n";
  std::exit(EXIT_FAILURE);
}

}  // namespace detail

// Shape rules of the selected kernel, checked without a GPU.
template <class Problem>
void validate_problem(const Problem& p) {
  alignas(16) static char dummy[16];
  bm_gemm_desc d = detail::make_desc(p, dummy, dummy, dummy);
  const int rc = bm_gemm_check(&d);
  if (rc == BM_ERR_TILE_DIVISIBILITY) {
    std::cerr << "Selected kernel requires M % CTA_M == 0, N % CTA_N == 0, K % CTA_K == 0\n";
    std::exit(EXIT_FAILURE);
  }
  if (rc != BM_OK) detail::die("problem rejected", rc);
}

inline void print_configuration() {
  std::printf("Selected MMA: tcgen05.mma kind::f16, FP32 accumulate in TMEM (variant %d: %s)\n",
              kVariant, kName);
  std::printf("Pipeline: 1 TMA producer warp, 1 MMA-issuer warp, 8 epilogue warps; "
              "strict tile check=%d\n", kStrictTiles ? 1 : 0);
}

// Prepare once, run `runner(launch, config)`, check the kernel status, release.
// `launch` must not outlive this call.
template <class Options, class Buffers, class Runner>
auto with_prepared(const Options& options, Buffers& buffers, const Runner& runner) {
  bm_gemm_desc d = detail::make_desc(options.problem, detail::device_pointer(buffers.d_A),
                                     detail::device_pointer(buffers.d_B),
                                     detail::device_pointer(buffers.d_C));
  bm_gemm_handle* h = nullptr;
  const int rc = bm_gemm_prepare(&d, &h);
  if (rc != BM_OK) detail::die("bm_gemm_prepare", rc);
  struct Release {
    bm_gemm_handle* h;
    ~Release() { bm_gemm_destroy(h); }
  } release{h};
  bm_launch_info info;
  bm_gemm_query(h, &info);
  gemm_bench::LaunchConfig config;
  config.smem_bytes = info.smem_bytes;
  config.grid = dim3(info.grid[0], info.grid[1], info.grid[2]);
  config.block = dim3(info.block[0], info.block[1], info.block[2]);
  config.cluster = dim3(info.cluster[0], info.cluster[1], info.cluster[2]);
  cudaStream_t stream = options.measurement.stream;
  auto launch = [h, stream]() {
    const int lrc = bm_gemm_launch(h, stream);
    if (lrc != BM_OK) detail::die("bm_gemm_launch", lrc);
  };
  // After the runner: every bounded wait inside the kernel must have been met.
  auto check_device = [h]() {
    uint32_t bits = 0;
    const int src = bm_gemm_status(h, &bits);
    if (src != BM_OK) {
      std::cerr << "Kernel status bits=0x" << std::hex << bits << std::dec << '\n';
      detail::die("bm_gemm_status", src);
    }
  };
  using Result = decltype(runner(launch, config));
  if constexpr (std::is_void_v<Result>) {
    runner(launch, config);
    check_device();
  } else {
    Result result = runner(launch, config);
    check_device();
    return result;
  }
}

}  // namespace gemm_backend
