// Diagonal scaling: C = diag(d) * B (row scale) and C = A * diag(b) (column
// scale).  Purely HBM-bound: one 4-byte read and one 4-byte write per element
// plus the (L2-resident) scale vector.  No tensor cores.
//
// Work unit: a "segment" of one row, 1024 float4 = 16 KiB, handled by one
// 256-thread CTA with four independent 128-bit streaming loads in flight per
// thread (evict-first hints: B and C are touched exactly once).  One CTA per
// segment lets the hardware scheduler balance the tail; at 8192 x 8192 that is
// 16384 CTAs, ~110 per SM.
//
// Multiplication is __fmul_rn: a single IEEE fp32 rounding and never fused,
// so the result is bit-identical to the reference kernels
// (src/dsl/codegen_cuda.py:1275-1307 kernel_diag_x_gen; diag_matmul.cpp:45-111).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "smm_host.h"

namespace smm {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int kSegVec = kThreads * kVecPerThread;  // float4 per segment

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ float4 scale4(float4 v, float s) {
  return make_float4(__fmul_rn(v.x, s), __fmul_rn(v.y, s), __fmul_rn(v.z, s), __fmul_rn(v.w, s));
}
__device__ __forceinline__ float4 mul4(float4 v, float4 s) {
  return make_float4(__fmul_rn(v.x, s.x), __fmul_rn(v.y, s.y), __fmul_rn(v.z, s.z), __fmul_rn(v.w, s.w));
}

// Row scale, 128-bit path: requires N % 4 == 0 and 16-byte aligned B, C.
__global__ void __launch_bounds__(kThreads) diag_rows_vec4(const float* __restrict__ d,
                                                           const float4* __restrict__ B, float4* __restrict__ C,
                                                           int n4, int segs_per_row) {
  const int row = blockIdx.x / segs_per_row;
  const int c0 = (blockIdx.x - row * segs_per_row) * kSegVec;
  const float s = __ldg(d + row);
  const long long base = static_cast<long long>(row) * n4;
  float4 v[kVecPerThread];
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n4) v[u] = ld_stream(B + base + c);
  }
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n4) st_stream(C + base + c, scale4(v[u], s));
  }
}

// Row scale, scalar path for any N / alignment.
__global__ void __launch_bounds__(kThreads) diag_rows_scalar(const float* __restrict__ d,
                                                             const float* __restrict__ B, float* __restrict__ C,
                                                             int n, int segs_per_row) {
  const int row = blockIdx.x / segs_per_row;
  const int c0 = (blockIdx.x - row * segs_per_row) * kSegVec;
  const float s = __ldg(d + row);
  const long long base = static_cast<long long>(row) * n;
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n) C[base + c] = __fmul_rn(__ldcs(B + base + c), s);
  }
}

// Column scale, 128-bit path.
__global__ void __launch_bounds__(kThreads) diag_cols_vec4(const float4* __restrict__ A,
                                                           const float4* __restrict__ b, float4* __restrict__ C,
                                                           int n4, int segs_per_row) {
  const int row = blockIdx.x / segs_per_row;
  const int c0 = (blockIdx.x - row * segs_per_row) * kSegVec;
  const long long base = static_cast<long long>(row) * n4;
  float4 v[kVecPerThread];
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n4) v[u] = ld_stream(A + base + c);
  }
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n4) st_stream(C + base + c, mul4(v[u], __ldg(b + c)));
  }
}

__global__ void __launch_bounds__(kThreads) diag_cols_scalar(const float* __restrict__ A,
                                                             const float* __restrict__ b, float* __restrict__ C,
                                                             int n, int segs_per_row) {
  const int row = blockIdx.x / segs_per_row;
  const int c0 = (blockIdx.x - row * segs_per_row) * kSegVec;
  const long long base = static_cast<long long>(row) * n;
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const int c = c0 + u * kThreads + threadIdx.x;
    if (c < n) C[base + c] = __fmul_rn(__ldcs(A + base + c), __ldg(b + c));
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_grid(long long rows, long long segs_per_row) {
  if (rows * segs_per_row > 0x7FFFFFFFLL)
    return set_error(SMM_ERR_INVALID, "diagonal scale: matrix too large for one launch (%lld segments)",
                     rows * segs_per_row);
  return SMM_OK;
}

int launch_rows(const float* d, const float* B, float* C, int M, int N, cudaStream_t st) {
  const bool vec = (N % 4 == 0) && aligned16(B) && aligned16(C);
  const int cols = vec ? N / 4 : N;
  const int segs = (cols + kSegVec - 1) / kSegVec;
  if (int rc = check_grid(M, segs)) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<long long>(M) * segs);
  if (vec)
    diag_rows_vec4<<<grid, kThreads, 0, st>>>(d, reinterpret_cast<const float4*>(B), reinterpret_cast<float4*>(C),
                                              cols, segs);
  else
    diag_rows_scalar<<<grid, kThreads, 0, st>>>(d, B, C, cols, segs);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "diag_rows launch");
  return SMM_OK;
}

}  // namespace
}  // namespace smm

using namespace smm;

extern "C" int smm_diag_rows(const float* d, const float* B, float* C, int M, int N, void* stream) {
  SMM_RANGE("smm_diag_rows");
  if (M < 0 || N < 0) return set_error(SMM_ERR_INVALID, "smm_diag_rows: negative shape %d x %d", M, N);
  if (M == 0 || N == 0) return SMM_OK;
  if (!d || !B || !C) return set_error(SMM_ERR_INVALID, "smm_diag_rows: null pointer");
  return launch_rows(d, B, C, M, N, as_stream(stream));
}

namespace smm {
namespace {
int launch_cols(const float* A, const float* b, float* C, int M, int N, cudaStream_t st) {
  const bool vec = (N % 4 == 0) && aligned16(A) && aligned16(b) && aligned16(C);
  const int cols = vec ? N / 4 : N;
  const int segs = (cols + kSegVec - 1) / kSegVec;
  if (int rc = check_grid(M, segs)) return rc;
  const unsigned grid = static_cast<unsigned>(static_cast<long long>(M) * segs);
  if (vec)
    diag_cols_vec4<<<grid, kThreads, 0, st>>>(reinterpret_cast<const float4*>(A), reinterpret_cast<const float4*>(b),
                                              reinterpret_cast<float4*>(C), cols, segs);
  else
    diag_cols_scalar<<<grid, kThreads, 0, st>>>(A, b, C, cols, segs);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "diag_cols launch");
  return SMM_OK;
}
}  // namespace
}  // namespace smm

extern "C" int smm_diag_cols(const float* A, const float* b, float* C, int M, int N, void* stream) {
  SMM_RANGE("smm_diag_cols");
  if (M < 0 || N < 0) return set_error(SMM_ERR_INVALID, "smm_diag_cols: negative shape %d x %d", M, N);
  if (M == 0 || N == 0) return SMM_OK;
  if (!A || !b || !C) return set_error(SMM_ERR_INVALID, "smm_diag_cols: null pointer");
  return launch_cols(A, b, C, M, N, as_stream(stream));
}

// ---------------------------------------------------------------- host-buffer path
namespace {
constexpr size_t kChunkBytes = size_t(32) << 20;  // rows per chunk: ~32 MiB of B

struct HostPipe {
  cudaStream_t st[2] = {nullptr, nullptr};
  cudaEvent_t d_ready = nullptr;
  bool init = false;
};

HostPipe& host_pipe(int dev) {  // dev in [0, 64)
  static HostPipe pipes[64];
  return pipes[dev];
}

size_t chunk_rows(int M, int N) {
  size_t row_bytes = static_cast<size_t>(N) * sizeof(float);
  size_t r = std::max<size_t>(1, kChunkBytes / std::max<size_t>(row_bytes, 1));
  return std::min<size_t>(r, static_cast<size_t>(M));
}

size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
}  // namespace

namespace {
// Host-buffer scale, rows (C = diag(d) B, d has M entries) or columns
// (C = A diag(b), b has N entries): the vector is copied once, then the
// matrix goes through in row chunks alternating between two streams.
size_t diag_host_ws(int M, int N, bool cols) {
  if (M <= 0 || N <= 0) return 0;
  const size_t rows = chunk_rows(M, N);
  const size_t chunk = round256(rows * static_cast<size_t>(N) * sizeof(float));
  return round256(static_cast<size_t>(cols ? N : M) * sizeof(float)) + 4 * chunk;  // vector + 2 x (in, out)
}

int diag_host(const char* who, bool cols, const float* v_host, const float* X_host, float* C_host, int M, int N,
              void* dev_ws, size_t ws_bytes) {
  if (M < 0 || N < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (M == 0 || N == 0) return SMM_OK;
  if (!v_host || !X_host || !C_host) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  const size_t need = diag_host_ws(M, N, cols);
  if (!dev_ws || ws_bytes < need)
    return set_error(SMM_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", who, ws_bytes, need);
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(SMM_ERR_UNSUPPORTED, "%s: device index %d >= 64", who, dev);
  HostPipe& hp = host_pipe(dev);
  {
    // first call on this device: create its streams (once, even when several
    // host threads make their first call together)
    static std::mutex init_mu;
    std::lock_guard<std::mutex> lock(init_mu);
    if (!hp.init) {
      for (auto& s : hp.st) SMM_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
      SMM_CUDA_TRY(cudaEventCreateWithFlags(&hp.d_ready, cudaEventDisableTiming), "event create");
      hp.init = true;
    }
  }
  const size_t rows = chunk_rows(M, N);
  const size_t chunk = round256(rows * static_cast<size_t>(N) * sizeof(float));
  const size_t vlen = static_cast<size_t>(cols ? N : M);
  uint8_t* ws = static_cast<uint8_t*>(dev_ws);
  float* v_dev = reinterpret_cast<float*>(ws);
  uint8_t* bufs = ws + round256(vlen * sizeof(float));
  float* bin[2] = {reinterpret_cast<float*>(bufs), reinterpret_cast<float*>(bufs + chunk)};
  float* cout[2] = {reinterpret_cast<float*>(bufs + 2 * chunk), reinterpret_cast<float*>(bufs + 3 * chunk)};

  SMM_CUDA_TRY(cudaMemcpyAsync(v_dev, v_host, sizeof(float) * vlen, cudaMemcpyHostToDevice, hp.st[0]),
               "copy scale vector");
  SMM_CUDA_TRY(cudaEventRecord(hp.d_ready, hp.st[0]), "event record");
  SMM_CUDA_TRY(cudaStreamWaitEvent(hp.st[1], hp.d_ready, 0), "stream wait");
  // Chunk c alternates between the two streams; within a stream the copy-in,
  // scale and copy-out of a chunk are ordered, and a buffer is reused only
  // after the previous copy-out on that stream (stream order).  Copies of one
  // stream overlap the kernel and opposite-direction copies of the other.
  int c = 0;
  for (size_t r0 = 0; r0 < static_cast<size_t>(M); r0 += rows, ++c) {
    const int k = c & 1;
    const size_t nr = std::min(rows, static_cast<size_t>(M) - r0);
    const size_t off = r0 * static_cast<size_t>(N);
    const size_t bytes = nr * static_cast<size_t>(N) * sizeof(float);
    SMM_CUDA_TRY(cudaMemcpyAsync(bin[k], X_host + off, bytes, cudaMemcpyHostToDevice, hp.st[k]), "copy chunk in");
    const int rc = cols ? launch_cols(bin[k], v_dev, cout[k], static_cast<int>(nr), N, hp.st[k])
                        : launch_rows(v_dev + r0, bin[k], cout[k], static_cast<int>(nr), N, hp.st[k]);
    if (rc) return rc;
    SMM_CUDA_TRY(cudaMemcpyAsync(C_host + off, cout[k], bytes, cudaMemcpyDeviceToHost, hp.st[k]), "copy chunk out");
  }
  for (auto& s : hp.st) SMM_CUDA_TRY(cudaStreamSynchronize(s), "stream sync");
  clear_error();
  return SMM_OK;
}
}  // namespace

extern "C" size_t smm_diag_rows_host_workspace_size(int M, int N) { return diag_host_ws(M, N, false); }

extern "C" int smm_diag_rows_host(const float* d_host, const float* B_host, float* C_host, int M, int N,
                                  void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_diag_rows_host");
  return diag_host("smm_diag_rows_host", false, d_host, B_host, C_host, M, N, dev_ws, ws_bytes);
}

extern "C" size_t smm_diag_cols_host_workspace_size(int M, int N) { return diag_host_ws(M, N, true); }

extern "C" int smm_diag_cols_host(const float* A_host, const float* b_host, float* C_host, int M, int N,
                                  void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_diag_cols_host");
  return diag_host("smm_diag_cols_host", true, b_host, A_host, C_host, M, N, dev_ws, ws_bytes);
}
