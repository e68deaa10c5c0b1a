// oracle/_ref wrapper around the reference's Toeplitz CPU kernel
// (toeplitz_matmul2.cpp:44-144, compute_matrix_multi1): Y = X*T with T
// (K x N) given by its generator g of length K+N-1, T[k][j] = g[(K-1)+(j-k)]
// (toeplitz_matmul2.cpp:35-42).  The earlier toeplitz_matmul.cpp kernel is
// numerically wrong and is not used.
//
// The left-side product C = T*B (T N x N, B N x ncols) is the transpose of
// B^T * T^T, and T^T is Toeplitz with generator gT[k] = g[2N-2-k].  The
// wrapper transposes B, reverses the generator, runs the reference kernel and
// transposes back, all outside the kernel's own chrono window.  The kernel
// accumulates with one FMA per k in ascending k.
//
// Tile configuration <64,64,64,4,16,1> is the driver's first sweep entry
// (toeplitz_matmul2.cpp:337).  Requires every dimension % 64 == 0.
#include "ref_wrap_common.h"
#include <vector>
#define main ref_toeplitz2_main
#include "toeplitz_matmul2.cpp"
#undef main

namespace {
constexpr int kBM = 64, kBN = 64, kBK = 64;

double run_right(float* X, float* gen, float* Y, int M, int N, int K) {
  // B cache holds a generator window of BK+BN-1 floats plus an 8-float
  // vector overrun; BK*BN floats covers it.
  refwrap::ThreadCaches caches((size_t)kBM * kBK, (size_t)kBK * kBN, (size_t)kBM * kBN);
  memset(Y, 0, sizeof(float) * (size_t)M * N);
  double gflops = 0.0, time_ms = 0.0;
  compute_matrix_multi1<kBM, kBN, kBK, 4, 16, 1, true, true, true>(X, gen, Y, M, N, K, gflops, time_ms,
                                                                   caches.c, caches.a, caches.b);
  return time_ms;
}
}  // namespace

extern "C" {

// The driver's own generator builder: g (K+N-1) of the K x N Toeplitz T.
void ref_toeplitz_compact(const float* T, float* g, int K, int N) {
  build_toeplitz_compact(const_cast<float*>(T), g, K, N);
}

// Right-side product as the driver runs it: Y(MxN) = X(MxK) * T(KxN).
double ref_toeplitz_right(const float* X, const float* gen, float* Y, int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || M % kBM || N % kBN || K % kBK) return -1.0;
  return run_right(const_cast<float*>(X), const_cast<float*>(gen), Y, M, N, K);
}

// Left-side product C(N x ncols) = T(NxN from gen[2N-1]) * B(N x ncols).
double ref_toeplitz_left(const float* gen, const float* B, float* C, int N, int ncols) {
  if (N <= 0 || ncols <= 0 || N % kBN || ncols % kBM) return -1.0;
  const long n = N;
  std::vector<float> Bt((size_t)ncols * N), gT(2 * (size_t)N - 1), Y((size_t)ncols * N);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < ncols; ++r)
    for (long k = 0; k < n; ++k) Bt[(size_t)r * n + k] = B[(size_t)k * ncols + r];
  for (long k = 0; k < 2 * n - 1; ++k) gT[k] = gen[2 * n - 2 - k];
  double ms = run_right(Bt.data(), gT.data(), Y.data(), ncols, N, N);
#pragma omp parallel for schedule(static)
  for (long c = 0; c < n; ++c)
    for (long r = 0; r < ncols; ++r) C[(size_t)c * ncols + r] = Y[(size_t)r * n + c];
  return ms;
}

}
