// Reference-compatible wrappers: one per operation the DSL's CUDA runner
// generates, with the generated wrapper's calling convention
//   <Out>_computation(lhs_data, rhs_data, out_data, gflops_out, n, time_ms_out)
// (src/dsl/codegen_cuda.py:44-45, 250-275 and the per-pair wrappers): device
// pointers, a square order n, synchronous on the legacy default stream, the
// kernels timed with CUDA events, and gflops counted as the generated
// wrappers do (2 n^3 for a product, n^2 for a diagonal scale or a sum).
// They run the primary entry points in the fp32 (3xTF32) mode; any workspace
// they need is allocated stream-ordered outside the timed window.  Unlike the
// generated wrappers they return a status instead of ignoring errors.
#include <cuda_runtime.h>

#include "smm_host.h"

namespace smm {
namespace {

template <typename F>
int compat_run(const char* who, float* gflops_out, float* time_ms_out, double flops, size_t ws_bytes, F&& call) {
  cudaStream_t st = nullptr;  // legacy default stream, as the generated wrappers use
  void* ws = nullptr;
  if (ws_bytes) SMM_CUDA_TRY(cudaMallocAsync(&ws, ws_bytes, st), "compat workspace allocation");
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaError_t ce = cudaEventCreate(&e0);
  if (ce == cudaSuccess) ce = cudaEventCreate(&e1);
  int rc = SMM_OK;
  if (ce == cudaSuccess) ce = cudaEventRecord(e0, st);
  if (ce == cudaSuccess) rc = call(ws, ws_bytes, st);
  if (ce == cudaSuccess) ce = cudaEventRecord(e1, st);
  if (ce == cudaSuccess) ce = cudaEventSynchronize(e1);
  float ms = 0.0f;
  if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, e0, e1);
  if (ws) cudaFreeAsync(ws, st);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (ce != cudaSuccess) return cuda_fail(ce, who);
  if (rc == SMM_OK) rc = smm_device_status(st);
  if (time_ms_out) *time_ms_out = ms;
  if (gflops_out) *gflops_out = ms > 0.0f ? static_cast<float>(flops * 1e-9 / (ms * 1e-3)) : 0.0f;
  return rc;
}

double cube(int n) { return 2.0 * n * static_cast<double>(n) * n; }
double square(int n) { return static_cast<double>(n) * n; }

}  // namespace
}  // namespace smm

using namespace smm;

#define SMM_COMPAT_MODE SMM_MODE_3XTF32

extern "C" int smm_compat_gen_x_gen(const float* A, const float* B, float* C, float* gflops_out, int n,
                                    float* time_ms_out) {
  SMM_RANGE("smm_compat_gen_x_gen");
  return compat_run("smm_compat_gen_x_gen", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_gemm_workspace_size(n, n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_gemm(A, B, C, n, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_diag_x_gen(const float* d, const float* B, float* C, float* gflops_out, int n,
                                     float* time_ms_out) {
  SMM_RANGE("smm_compat_diag_x_gen");
  return compat_run("smm_compat_diag_x_gen", gflops_out, time_ms_out, square(n), 0,
                    [&](void*, size_t, cudaStream_t st) { return smm_diag_rows(d, B, C, n, n, st); });
}

extern "C" int smm_compat_gen_x_diag(const float* A, const float* d, float* C, float* gflops_out, int n,
                                     float* time_ms_out) {
  SMM_RANGE("smm_compat_gen_x_diag");
  return compat_run("smm_compat_gen_x_diag", gflops_out, time_ms_out, square(n), 0,
                    [&](void*, size_t, cudaStream_t st) { return smm_diag_cols(A, d, C, n, n, st); });
}

extern "C" int smm_compat_upper_x_gen(const float* U, const float* B, float* C, float* gflops_out, int n,
                                      float* time_ms_out) {
  SMM_RANGE("smm_compat_upper_x_gen");
  return compat_run("smm_compat_upper_x_gen", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_upper_left_workspace_size(n, n, SMM_FMT_PACKED, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_upper_left(U, SMM_FMT_PACKED, B, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_toeplitz_x_gen(const float* g, const float* B, float* C, float* gflops_out, int n,
                                         float* time_ms_out) {
  SMM_RANGE("smm_compat_toeplitz_x_gen");
  return compat_run("smm_compat_toeplitz_x_gen", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_toeplitz_left_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_toeplitz_left(g, B, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_symm_x_gen(const float* S, const float* B, float* C, float* gflops_out, int n,
                                     float* time_ms_out) {
  SMM_RANGE("smm_compat_symm_x_gen");
  return compat_run("smm_compat_symm_x_gen", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_symm_left_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_symm_left(S, B, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_gen_x_symm(const float* A, const float* S, float* C, float* gflops_out, int n,
                                     float* time_ms_out) {
  SMM_RANGE("smm_compat_gen_x_symm");
  return compat_run("smm_compat_gen_x_symm", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_gen_x_struct_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_gen_x_symm(A, S, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_gen_x_upper(const float* A, const float* U, float* C, float* gflops_out, int n,
                                      float* time_ms_out) {
  SMM_RANGE("smm_compat_gen_x_upper");
  return compat_run("smm_compat_gen_x_upper", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_gen_x_struct_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_gen_x_upper(A, U, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_symm_x_symm(const float* S1, const float* S2, float* C, float* gflops_out, int n,
                                      float* time_ms_out) {
  SMM_RANGE("smm_compat_symm_x_symm");
  return compat_run("smm_compat_symm_x_symm", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_symm_x_symm_workspace_size(n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_symm_x_symm_ws(S1, S2, C, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_gen_x_lower(const float* A, const float* L, float* C, float* gflops_out, int n,
                                      float* time_ms_out) {
  SMM_RANGE("smm_compat_gen_x_lower");
  return compat_run("smm_compat_gen_x_lower", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_gen_x_struct_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_gen_x_lower(A, L, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_lower_x_gen(const float* L, const float* B, float* C, float* gflops_out, int n,
                                      float* time_ms_out) {
  SMM_RANGE("smm_compat_lower_x_gen");
  return compat_run("smm_compat_lower_x_gen", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_lower_left_workspace_size(n, n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_lower_left(L, B, C, n, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_lower_x_lower(const float* L1, const float* L2, float* C, float* gflops_out, int n,
                                        float* time_ms_out) {
  SMM_RANGE("smm_compat_lower_x_lower");
  return compat_run("smm_compat_lower_x_lower", gflops_out, time_ms_out, cube(n),
                    n > 0 ? smm_lower_x_lower_workspace_size(n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_lower_x_lower_ws(L1, L2, C, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}

extern "C" int smm_compat_add_gen_symm(const float* A, const float* S, float* C, float* gflops_out, int n,
                                       float* time_ms_out) {
  SMM_RANGE("smm_compat_add_gen_symm");
  return compat_run("smm_compat_add_gen_symm", gflops_out, time_ms_out, square(n), 0,
                    [&](void*, size_t, cudaStream_t st) { return smm_add_struct(A, S, SMM_STRUCT_SYMM, C, n, st); });
}

extern "C" int smm_compat_symm_sandwich(const float* A, const float* S, const float* B, float* C, float* gflops_out,
                                        int n, float* time_ms_out) {
  SMM_RANGE("smm_compat_symm_sandwich");
  return compat_run("smm_compat_symm_sandwich", gflops_out, time_ms_out, 2.0 * cube(n),
                    n > 0 ? smm_symm_sandwich_workspace_size(n, SMM_COMPAT_MODE) : 0,
                    [&](void* ws, size_t wb, cudaStream_t st) {
                      return smm_symm_sandwich(A, S, B, C, n, SMM_COMPAT_MODE, ws, wb, st);
                    });
}
