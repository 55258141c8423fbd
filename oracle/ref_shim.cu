// ref_shim.cu - exposes the reference's own CPU code through a C ABI.
//
// TEST INFRASTRUCTURE ONLY. Compiled by oracle/Makefile against the
// reference's unmodified headers, included from where they lie
// (host/validation.cuh, which includes host/common.cuh), into
// oracle/_ref/libbm_ref.so. It is used to pin the C oracle
// (oracle/bm_oracle.c) and as the "reference" CPU baseline of bench.py.
// Nothing here runs on a GPU: only make_input_value, GemmProblem's index
// functions and reference_gemm_entry are called.
#include "host/validation.cuh"

#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

struct RefState {
  gemm_bench::GemmProblem problem;
  thrust::host_vector<gemm_bench::Element> A, B;
};

}  // namespace

extern "C" {

// Inputs exactly as gemm_bench::GemmBuffers builds them on the host
// (host/common.cuh:129-140): srand(0), then make_input_value over A, then B.
void* bmref_create(int m, int n, int k, char ta, char tb, int mode) {
  auto* s = new RefState();
  s->problem.m = m;
  s->problem.n = n;
  s->problem.k = k;
  s->problem.transA = ta;
  s->problem.transB = tb;
  s->A.resize(s->problem.a_elements());
  s->B.resize(s->problem.b_elements());
  std::srand(0);
  const auto im = static_cast<gemm_bench::InputMode>(mode);
  for (std::size_t i = 0; i < s->A.size(); ++i) s->A[i] = gemm_bench::make_input_value(i, 0, im);
  for (std::size_t i = 0; i < s->B.size(); ++i) s->B[i] = gemm_bench::make_input_value(i, 1, im);
  return s;
}

// Same problem with caller-provided FP16 bit patterns (for inputs the
// reference cannot generate, e.g. uniform[-1,1]).
void* bmref_create_from(int m, int n, int k, char ta, char tb, const uint16_t* a,
                        const uint16_t* b) {
  auto* s = new RefState();
  s->problem.m = m;
  s->problem.n = n;
  s->problem.k = k;
  s->problem.transA = ta;
  s->problem.transB = tb;
  s->A.resize(s->problem.a_elements());
  s->B.resize(s->problem.b_elements());
  std::memcpy(s->A.data(), a, s->A.size() * sizeof(uint16_t));
  std::memcpy(s->B.data(), b, s->B.size() * sizeof(uint16_t));
  return s;
}

void bmref_export(void* h, uint16_t* a, uint16_t* b) {
  auto* s = static_cast<RefState*>(h);
  std::memcpy(a, s->A.data(), s->A.size() * sizeof(uint16_t));
  std::memcpy(b, s->B.data(), s->B.size() * sizeof(uint16_t));
}

int64_t bmref_a_index(void* h, int row, int p) {
  return static_cast<int64_t>(static_cast<RefState*>(h)->problem.a_index(row, p));
}
int64_t bmref_b_index(void* h, int col, int p) {
  return static_cast<int64_t>(static_cast<RefState*>(h)->problem.b_index(col, p));
}
int64_t bmref_c_index(void* h, int row, int col) {
  return static_cast<int64_t>(static_cast<RefState*>(h)->problem.c_index(row, col));
}

double bmref_entry(void* h, int row, int col) {
  auto* s = static_cast<RefState*>(h);
  return gemm_bench::reference_gemm_entry(s->problem, s->A, s->B, row, col);
}

// reference_gemm_entry over (rows[i], cols[i]), i < count, on `threads`
// std::threads (the function is pure).
void bmref_entries(void* h, const int* rows, const int* cols, int64_t count, double* out,
                   int threads) {
  auto* s = static_cast<RefState*>(h);
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const int64_t b = count * t / threads, e = count * (t + 1) / threads;
    pool.emplace_back([s, rows, cols, out, b, e] {
      for (int64_t i = b; i < e; ++i)
        out[i] = gemm_bench::reference_gemm_entry(s->problem, s->A, s->B, rows[i], cols[i]);
    });
  }
  for (auto& th : pool) th.join();
}

void bmref_destroy(void* h) { delete static_cast<RefState*>(h); }

}  // extern "C"
