// oracle/_ref wrapper around the reference's dense CPU GEMM kernel
// (gemm_benchmark.cpp:40-156, compute_matrix_multi1).  Tile configuration
// <64,64,64,8,8,1> is one of the driver's own sweep entries
// (gemm_benchmark.cpp:330).  Requires M, N, K all multiples of 64 (the
// divisible specialisation; the non-divisible one reads stale cache entries).
#include "ref_wrap_common.h"
#define main ref_gemm_benchmark_main
#include "gemm_benchmark.cpp"
#undef main

extern "C" {

// C = A(MxK) * B(KxN), row-major fp32.  Returns the kernel's own time in ms,
// or -1 when the shape is not divisible by the tile configuration.
double ref_gemm(const float* A, const float* B, float* C, int M, int N, int K) {
  constexpr int BM = 64, BN = 64, BK = 64;
  if (M <= 0 || N <= 0 || K <= 0 || M % BM || N % BN || K % BK) return -1.0;
  refwrap::ThreadCaches caches((size_t)BM * BK, (size_t)BK * BN, (size_t)BM * BN);
  memset(C, 0, sizeof(float) * (size_t)M * N);
  double gflops = 0.0, time_ms = 0.0;
  compute_matrix_multi1<BM, BN, BK, 8, 8, 1, true, true, true>(
      const_cast<float*>(A), const_cast<float*>(B), C, M, N, K, gflops, time_ms,
      caches.c, caches.a, caches.b);
  return time_ms;
}

}
