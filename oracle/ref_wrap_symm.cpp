// oracle/_ref wrapper around the reference's symmetric CPU kernel
// (symmetric_matmul.cpp:84-211, compute_matrix_multi1): W = A*S with S
// packed upper (idx(i,j) = i(2K-i+1)/2 + (j-i) for i <= j,
// symmetric_matmul.cpp:47-50) and mirrored while the B cache is filled
// (symmetric_matmul.cpp:131-157).  That fill exists only in the divisible
// specialisation, so N%BN == K%BK == 0 is required.
//
// The driver's main() references an undeclared variable `check_results`
// (symmetric_matmul.cpp:393, :400) and does not compile as shipped; a
// file-scope bool of that name, declared before the include, lets main()
// compile (function parameters of the same name shadow it).  main() itself is
// renamed and never called.
//
// The sandwich C = A*S*B runs this kernel, then the dense GEMM kernel of
// gemm_benchmark.cpp (exported from libref_gemm.so) on W*B.
#include "ref_wrap_common.h"
#include <vector>
static bool check_results = false;
#define main ref_symmetric_main
#include "symmetric_matmul.cpp"
#undef main

namespace {
constexpr int kBM = 64, kBN = 64, kBK = 64;
}

extern "C" {

// W(MxN) = A(MxK) * S(KxK packed upper) with N == K.  Requires M,N % 64 == 0.
double ref_symm_right(const float* A, const float* S_packed, float* W, int M, int N) {
  if (M <= 0 || N <= 0 || M % kBM || N % kBN) return -1.0;
  refwrap::ThreadCaches caches((size_t)kBM * kBK, (size_t)kBK * kBN, (size_t)kBM * kBN);
  memset(W, 0, sizeof(float) * (size_t)M * N);
  double gflops = 0.0, time_ms = 0.0;
  compute_matrix_multi1<kBM, kBN, kBK, 8, 8, 1, true, true, true>(
      const_cast<float*>(A), S_packed, W, M, N, N, gflops, time_ms, caches.c, caches.a, caches.b);
  return time_ms;
}

}
