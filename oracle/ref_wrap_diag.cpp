// oracle/_ref wrapper around the reference's diagonal-scaling CPU kernel
// (diag_matmul.cpp:45-111, optimized_compute), which computes the column
// scale C = A*diag(b).  The row scale C = diag(d)*B is its transpose:
// diag(d)*B = (B^T * diag(d))^T, one fp32 multiply per element either way,
// so the result is bit-identical.  The transposes sit outside the kernel's
// own chrono window.  Tile configuration <64,64,8,8> is the first entry of
// the driver's own sweep (diag_matmul.cpp:273).
#include "ref_wrap_common.h"
#include <vector>
#define main ref_diag_matmul_main
#include "diag_matmul.cpp"
#undef main

namespace {
constexpr int kBM = 64, kBD = 64;

double run_colscale(const float* A, const float* b, float* C, int M, int N) {
  int nt = omp_get_max_threads();
  long pg = sysconf(_SC_PAGESIZE);
  std::vector<float*> abuf(nt), bbuf(nt);
  for (int t = 0; t < nt; ++t) {
    abuf[t] = (float*)aligned_alloc(pg, ((kBM * kBD * sizeof(float) + pg - 1) / pg) * pg);
    bbuf[t] = (float*)aligned_alloc(pg, ((kBD * sizeof(float) + pg - 1) / pg) * pg);
  }
  double gflops = 0.0, time_ms = 0.0;
  if (M % kBM == 0 && N % kBD == 0)
    optimized_compute<kBM, kBD, 8, 8, true, true>(A, b, C, M, N, gflops, time_ms, abuf.data(), bbuf.data());
  else
    optimized_compute<kBM, kBD, 8, 8, false, false>(A, b, C, M, N, gflops, time_ms, abuf.data(), bbuf.data());
  for (int t = 0; t < nt; ++t) {
    free(abuf[t]);
    free(bbuf[t]);
  }
  return time_ms;
}

void transpose(const float* src, float* dst, int rows, int cols) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < cols; ++j) dst[(size_t)j * rows + i] = src[(size_t)i * cols + j];
}
}  // namespace

extern "C" {

// Column scale exactly as the driver runs it: C[i][j] = A[i][j] * b[j].
double ref_diag_cols(const float* A, const float* b, float* C, int M, int N) {
  if (M <= 0 || N <= 0 || M % kBM || N % kBD) return -1.0;
  return run_colscale(A, b, C, M, N);
}

// Row scale C[i][j] = d[i] * B[i][j] (M rows, N columns) through the column
// kernel on B^T.  Returns the kernel's own time in ms.
double ref_diag_rows(const float* d, const float* B, float* C, int M, int N) {
  if (M <= 0 || N <= 0 || M % kBM || N % kBD) return -1.0;
  std::vector<float> Bt((size_t)M * N), Ct((size_t)M * N);
  transpose(B, Bt.data(), M, N);
  double ms = run_colscale(Bt.data(), d, Ct.data(), N, M);
  transpose(Ct.data(), C, N, M);
  return ms;
}

}
