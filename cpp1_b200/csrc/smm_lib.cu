// libsmm host library: C ABI entry points for the tensor-core contractions
// (dense GEMM, upper-triangular-left, Toeplitz-left, symmetric-left and the
// symmetric sandwich), error/status plumbing and TMA descriptor encoding.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "smm_host.h"
#include "smm_umma.cuh"

// Sticky kernel status word, one per device context.
__device__ uint32_t g_smm_status;

namespace smm {

// ---------------------------------------------------------------- errors
namespace {
thread_local char t_last_error[512] = "";
std::atomic<unsigned long long> g_launches{0};
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}
void clear_error() { t_last_error[0] = '\0'; }
int cuda_fail(cudaError_t e, const char* what) {
  return set_error(SMM_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}
void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

uint32_t* device_status_word() {
  static uint32_t* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev & 63]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_smm_status) != cudaSuccess) return nullptr;
    addr[dev & 63] = static_cast<uint32_t*>(p);
  }
  return addr[dev & 63];
}

unsigned long long wait_limit_ns() {
  static unsigned long long v = [] {
    const char* e = std::getenv("SMM_WAIT_LIMIT_MS");
    unsigned long long ms = e ? std::strtoull(e, nullptr, 10) : 2000ull;
    if (ms == 0) ms = 2000ull;
    return ms * 1000000ull;
  }();
  return v;
}

// ---------------------------------------------------------------- TMA maps
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 2-D fp32 tensor map over a row-major matrix (rows x cols, leading dimension
// ld elements), box of box_cols x box_rows elements.
int make_tmap(CUtensorMap* m, const float* base, int rows, int cols, int ld, int box_cols, int box_rows,
              CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return set_error(SMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * sizeof(float)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %d x %d (ld %d)", int(r), rows, cols, ld);
  return SMM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
int round4(int x) { return (x + 3) & ~3; }

// ---------------------------------------------------------------- pad copy
// dst (rows x ld_dst) = src (rows x cols, ld_src) with zero columns appended.
__global__ void pad_cols_kernel(const float* __restrict__ src, int rows, int cols, int ld_src,
                                float* __restrict__ dst, int ld_dst) {
  const long long total = static_cast<long long>(rows) * ld_dst;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / ld_dst;
    const int c = static_cast<int>(i - r * ld_dst);
    dst[i] = c < cols ? src[r * ld_src + c] : 0.0f;
  }
}

int pad_copy(const float* src, int rows, int cols, float* dst, int ld_dst, cudaStream_t st) {
  const long long total = static_cast<long long>(rows) * ld_dst;
  const int grid = static_cast<int>(std::min<long long>((total + 255) / 256, 148LL * 16));
  pad_cols_kernel<<<std::max(grid, 1), 256, 0, st>>>(src, rows, cols, cols, dst, ld_dst);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "pad copy launch");
  return SMM_OK;
}

// ---------------------------------------------------------------- launches
template <AKind AK, BKind BK, bool SPLIT3, int BN, int STAGES>
int launch_umma(const CUtensorMap& ta, const CUtensorMap& tb, const UmmaParams& p, cudaStream_t st) {
  auto kern = umma_gemm_kernel<AK, BK, SPLIT3, BN, STAGES>;
  constexpr int smem = umma_smem_bytes<BN, SPLIT3, STAGES>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static bool attr_set[64] = {};
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (!attr_set[dev & 63]) {
    SMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute(max dynamic smem)");
    attr_set[dev & 63] = true;
  }
  dim3 grid(p.col_tiles, p.row_tiles);
  kern<<<grid, kThreads, smem, st>>>(ta, tb, p);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "tcgen05 contraction launch");
  return SMM_OK;
}

// Stage counts fill ~192 KiB of shared memory.
template <AKind AK, BKind BK, int BN>
int launch_mode(bool split3, const CUtensorMap& ta, const CUtensorMap& tb, const UmmaParams& p, cudaStream_t st) {
  if constexpr (BN <= 128) {
    if (split3) {
      constexpr int S = (BN == 128) ? 6 : 8;
      return launch_umma<AK, BK, true, BN, S>(ta, tb, p, st);
    }
  } else {
    if (split3) return set_error(SMM_ERR_INVALID, "3xTF32 tiles are at most 128 columns wide");
  }
  constexpr int S = 8;
  return launch_umma<AK, BK, false, BN, S>(ta, tb, p, st);
}

template <AKind AK, BKind BK>
int launch_bn(int bn, bool split3, const CUtensorMap& ta, const CUtensorMap& tb, const UmmaParams& p,
              cudaStream_t st) {
  switch (bn) {
    case 256: return launch_mode<AK, BK, 256>(split3, ta, tb, p, st);
    case 128: return launch_mode<AK, BK, 128>(split3, ta, tb, p, st);
    default: return launch_mode<AK, BK, 64>(split3, ta, tb, p, st);
  }
}

// Output tile width: the widest tile that still yields about a wave of CTAs.
int pick_bn(int M, int N) {
  const long long rt = (M + kBM - 1) / kBM;
  const char* e = std::getenv("SMM_TILE_N");
  if (e) {
    int v = std::atoi(e);
    if (v == 64 || v == 128 || v == 256) return v;
  }
  if (N > 128 && rt * ((N + 255) / 256) >= 120) return 256;
  if (N > 64 && rt * ((N + 127) / 128) >= 100) return 128;
  return 64;
}

// Diagnostic record target for the next contraction launch (set by
// smm_debug_trace_next, consumed by one launch).
thread_local uint32_t* g_trace = nullptr;

bool valid_mode(int mode) { return mode == SMM_MODE_3XTF32 || mode == SMM_MODE_TF32 || mode == SMM_MODE_BF16; }

// Core contraction: C(M x N, ldc) = Aop(M x K) * B(K x N, ldb).
// Preconditions: B (and A when dense) 16-byte aligned with ld % 4 == 0.
// Operand description for run_contraction: a dense TMA-loaded matrix (ptr,
// ld) or a structured one (src, dim, row0).
struct Operand {
  const float* ptr = nullptr;
  int ld = 0;
  const float* src = nullptr;
  int dim = 0;
  int row0 = 0;
};

int run_contraction(AKind ak, BKind bk, int mode, const Operand& a, const Operand& b, float* C, int ldc, int M,
                    int N, int K, cudaStream_t st) {
  if (mode == SMM_MODE_BF16) return set_error(SMM_ERR_UNSUPPORTED, "bf16 mode not built for this operation");
  const bool split3 = (mode == SMM_MODE_3XTF32);
  // 3xTF32 keeps two chunk accumulators and a running sum in tensor memory
  // (3 x BN of its 512 columns), so its tiles are at most 128 wide.
  const int bn = split3 ? std::min(pick_bn(M, N), 128) : pick_bn(M, N);
  CUtensorMap tb{}, ta{};
  const bool a_tma = (ak == AKind::Dense || ak == AKind::UpperDense);
  const bool b_tma = (bk == BKind::Dense);
  if (b_tma) {
    if (int rc = make_tmap(&tb, b.ptr, K, N, b.ld, 32, 16, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)) return rc;
  }
  if (a_tma) {
    if (int rc = make_tmap(&ta, a.ptr, M, K, a.ld, 16, 128, CU_TENSOR_MAP_SWIZZLE_64B)) return rc;
  }
  UmmaParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.a_src = a.src;
  p.a_dim = a.dim;
  p.a_row0 = a.row0;
  p.b_src = b.src;
  p.b_dim = b.dim;
  p.row_tiles = (M + kBM - 1) / kBM;
  p.col_tiles = (N + bn - 1) / bn;
  p.status = device_status_word();
  p.wait_limit_ns = wait_limit_ns();
  p.trace = g_trace;
  if (!p.status) return set_error(SMM_ERR_CUDA, "device status word unavailable");
  if (p.row_tiles > 65535) return set_error(SMM_ERR_INVALID, "M = %d too large (max %d)", M, 65535 * kBM);
  g_trace = nullptr;
  if (bk == BKind::Dense) {
    switch (ak) {
      case AKind::Dense: return launch_bn<AKind::Dense, BKind::Dense>(bn, split3, ta, tb, p, st);
      case AKind::UpperDense: return launch_bn<AKind::UpperDense, BKind::Dense>(bn, split3, ta, tb, p, st);
      case AKind::UpperPacked: return launch_bn<AKind::UpperPacked, BKind::Dense>(bn, split3, ta, tb, p, st);
      case AKind::Toeplitz: return launch_bn<AKind::Toeplitz, BKind::Dense>(bn, split3, ta, tb, p, st);
      case AKind::SymmPacked: return launch_bn<AKind::SymmPacked, BKind::Dense>(bn, split3, ta, tb, p, st);
    }
  }
  if (ak == AKind::Dense && bk == BKind::UpperPacked)
    return launch_bn<AKind::Dense, BKind::UpperPacked>(bn, split3, ta, tb, p, st);
  if (ak == AKind::Dense && bk == BKind::SymmPacked)
    return launch_bn<AKind::Dense, BKind::SymmPacked>(bn, split3, ta, tb, p, st);
  if (ak == AKind::SymmPacked && bk == BKind::SymmPacked)
    return launch_bn<AKind::SymmPacked, BKind::SymmPacked>(bn, split3, ta, tb, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

Operand dense_op(const float* ptr, int ld) {
  Operand o;
  o.ptr = ptr;
  o.ld = ld;
  return o;
}
Operand structured_op(const float* src, int dim, int row0 = 0) {
  Operand o;
  o.src = src;
  o.dim = dim;
  o.row0 = row0;
  return o;
}

// A right operand (rows x cols row-major) usable by TMA: either the caller's
// array or a padded copy in the workspace.
struct Staged {
  const float* ptr;
  int ld;
};

bool needs_pad(const float* p, int cols) { return (cols % 4 != 0) || !aligned16(p); }
size_t pad_bytes(const float* p, int rows, int cols) {
  return needs_pad(p, cols) ? round256(static_cast<size_t>(rows) * round4(cols) * sizeof(float)) : 0;
}

int stage_operand(const float* src, int rows, int cols, uint8_t*& ws_cur, Staged* out, cudaStream_t st) {
  if (!needs_pad(src, cols)) {
    *out = {src, cols};
    return SMM_OK;
  }
  float* dst = reinterpret_cast<float*>(ws_cur);
  const int ld = round4(cols);
  if (int rc = pad_copy(src, rows, cols, dst, ld, st)) return rc;
  ws_cur += round256(static_cast<size_t>(rows) * ld * sizeof(float));
  *out = {dst, ld};
  return SMM_OK;
}

int check_ws(const char* who, void* ws, size_t have, size_t need) {
  if (need == 0) return SMM_OK;
  if (!ws || have < need)
    return set_error(SMM_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu required", who, have, need);
  if (!aligned16(ws)) return set_error(SMM_ERR_WORKSPACE, "%s: workspace must be 16-byte aligned", who);
  return SMM_OK;
}

int zero_output(float* C, int rows, int cols, cudaStream_t st) {
  SMM_CUDA_TRY(cudaMemsetAsync(C, 0, sizeof(float) * static_cast<size_t>(rows) * cols, st), "zero output");
  return SMM_OK;
}

}  // namespace
}  // namespace smm

using namespace smm;

// ---------------------------------------------------------------- C ABI
extern "C" const char* smm_last_error(void) { return t_last_error; }
extern "C" int smm_version(void) { return 100; }  // 0.1.0
extern "C" unsigned long long smm_launch_count(void) { return g_launches.load(); }

extern "C" int smm_device_status(void* stream) {
  uint32_t* w = device_status_word();
  if (!w) return set_error(SMM_ERR_CUDA, "device status word unavailable");
  SMM_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)), "stream synchronize");
  uint32_t v = 0;
  SMM_CUDA_TRY(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost), "read status word");
  if (v) {
    SMM_CUDA_TRY(cudaMemset(w, 0, sizeof(v)), "clear status word");
    if (v & kDevErrTimeout)
      return set_error(SMM_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait expired (status 0x%x); it exited cleanly", v);
  }
  return SMM_OK;
}

extern "C" size_t smm_gemm_workspace_size(int M, int N, int K, int mode) {
  (void)mode;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // Conservative: assumes both operands need a padded copy unless the shape
  // alone guarantees they do not (pointer alignment is not known here).
  size_t b = 0;
  b += round256(static_cast<size_t>(M) * round4(K) * sizeof(float));
  b += round256(static_cast<size_t>(K) * round4(N) * sizeof(float));
  return b;
}

extern "C" int smm_gemm(const float* A, const float* B, float* C, int M, int N, int K, int mode, void* ws,
                        size_t ws_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "smm_gemm: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_gemm: unknown mode %d", mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(SMM_ERR_INVALID, "smm_gemm: null pointer");
  cudaStream_t st = as_stream(stream);
  if (K == 0) return zero_output(C, M, N, st);
  const size_t need = pad_bytes(A, M, K) + pad_bytes(B, K, N);
  if (int rc = check_ws("smm_gemm", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a, b;
  if (int rc = stage_operand(A, M, K, cur, &a, st)) return rc;
  if (int rc = stage_operand(B, K, N, cur, &b, st)) return rc;
  return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, a.ld), dense_op(b.ptr, b.ld), C, N, M, N, K,
                         st);
}

extern "C" size_t smm_upper_left_workspace_size(int N, int ncols, int u_fmt, int mode) {
  (void)mode;
  if (N <= 0 || ncols <= 0) return 0;
  size_t b = round256(static_cast<size_t>(N) * round4(ncols) * sizeof(float));
  if (u_fmt == SMM_FMT_DENSE) b += round256(static_cast<size_t>(N) * round4(N) * sizeof(float));
  return b;
}

namespace {
int check_slab(const char* who, int N, int ncols, int row0, int nrows) {
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
    return set_error(SMM_ERR_INVALID, "%s: bad shape N=%d ncols=%d rows [%d, %d)", who, N, ncols, row0, row0 + nrows);
  return SMM_OK;
}
}  // namespace

extern "C" int smm_upper_left_rows(const float* U, int u_fmt, const float* B, float* C, int N, int ncols, int row0,
                                   int nrows, int mode, void* ws, size_t ws_bytes, void* stream) {
  if (int rc = check_slab("smm_upper_left", N, ncols, row0, nrows)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_upper_left: unknown mode %d", mode);
  if (u_fmt != SMM_FMT_PACKED && u_fmt != SMM_FMT_DENSE)
    return set_error(SMM_ERR_INVALID, "smm_upper_left: unknown U format %d", u_fmt);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!U || !B || !C) return set_error(SMM_ERR_INVALID, "smm_upper_left: null pointer");
  cudaStream_t st = as_stream(stream);
  size_t need = pad_bytes(B, N, ncols);
  if (u_fmt == SMM_FMT_DENSE) need += pad_bytes(U, N, N);
  if (int rc = check_ws("smm_upper_left", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, cur, &b, st)) return rc;
  if (u_fmt == SMM_FMT_DENSE) {
    Staged u;
    if (int rc = stage_operand(U, N, N, cur, &u, st)) return rc;
    const float* urows = u.ptr + static_cast<size_t>(row0) * u.ld;
    Operand ua = dense_op(urows, u.ld);
    ua.dim = N;
    ua.row0 = row0;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ua, dense_op(b.ptr, b.ld), C, ncols, nrows, ncols,
                           N, st);
  }
  return run_contraction(AKind::UpperPacked, BKind::Dense, mode, structured_op(U, N, row0), dense_op(b.ptr, b.ld), C,
                         ncols, nrows, ncols, N, st);
}

extern "C" int smm_upper_left(const float* U, int u_fmt, const float* B, float* C, int N, int ncols, int mode,
                              void* ws, size_t ws_bytes, void* stream) {
  return smm_upper_left_rows(U, u_fmt, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

extern "C" size_t smm_toeplitz_left_workspace_size(int N, int ncols, int mode) {
  (void)mode;
  if (N <= 0 || ncols <= 0) return 0;
  return round256(static_cast<size_t>(N) * round4(ncols) * sizeof(float));
}

extern "C" int smm_toeplitz_left_rows(const float* g, const float* B, float* C, int N, int ncols, int row0,
                                      int nrows, int mode, void* ws, size_t ws_bytes, void* stream) {
  if (int rc = check_slab("smm_toeplitz_left", N, ncols, row0, nrows)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_toeplitz_left: unknown mode %d", mode);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!g || !B || !C) return set_error(SMM_ERR_INVALID, "smm_toeplitz_left: null pointer");
  cudaStream_t st = as_stream(stream);
  if (int rc = check_ws("smm_toeplitz_left", ws, ws_bytes, pad_bytes(B, N, ncols))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, cur, &b, st)) return rc;
  return run_contraction(AKind::Toeplitz, BKind::Dense, mode, structured_op(g, N, row0), dense_op(b.ptr, b.ld), C,
                         ncols, nrows, ncols, N, st);
}

extern "C" int smm_toeplitz_left(const float* g, const float* B, float* C, int N, int ncols, int mode, void* ws,
                                 size_t ws_bytes, void* stream) {
  return smm_toeplitz_left_rows(g, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

extern "C" size_t smm_symm_left_workspace_size(int N, int ncols, int mode) {
  return smm_toeplitz_left_workspace_size(N, ncols, mode);
}

extern "C" int smm_symm_left_rows(const float* S, const float* B, float* C, int N, int ncols, int row0, int nrows,
                                  int mode, void* ws, size_t ws_bytes, void* stream) {
  if (int rc = check_slab("smm_symm_left", N, ncols, row0, nrows)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_left: unknown mode %d", mode);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_left: null pointer");
  cudaStream_t st = as_stream(stream);
  if (int rc = check_ws("smm_symm_left", ws, ws_bytes, pad_bytes(B, N, ncols))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, cur, &b, st)) return rc;
  return run_contraction(AKind::SymmPacked, BKind::Dense, mode, structured_op(S, N, row0), dense_op(b.ptr, b.ld), C,
                         ncols, nrows, ncols, N, st);
}

extern "C" int smm_symm_left(const float* S, const float* B, float* C, int N, int ncols, int mode, void* ws,
                             size_t ws_bytes, void* stream) {
  return smm_symm_left_rows(S, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

extern "C" size_t smm_symm_sandwich_workspace_size(int N, int mode) {
  (void)mode;
  if (N <= 0) return 0;
  const size_t mat = round256(static_cast<size_t>(N) * round4(N) * sizeof(float));
  return 3 * mat;  // X = S B (padded stride), plus padded copies of A and B when needed
}

extern "C" int smm_symm_sandwich(const float* A, const float* S, const float* B, float* C, int N, int mode,
                                 void* ws, size_t ws_bytes, void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!A || !S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: null pointer");
  cudaStream_t st = as_stream(stream);
  const int ldx = round4(N);
  const size_t xbytes = round256(static_cast<size_t>(N) * ldx * sizeof(float));
  const size_t need = xbytes + pad_bytes(A, N, N) + pad_bytes(B, N, N);
  if (int rc = check_ws("smm_symm_sandwich", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* X = reinterpret_cast<float*>(cur);
  cur += xbytes;
  Staged a, b;
  if (int rc = stage_operand(A, N, N, cur, &a, st)) return rc;
  if (int rc = stage_operand(B, N, N, cur, &b, st)) return rc;
  if (ldx != N) SMM_CUDA_TRY(cudaMemsetAsync(X, 0, xbytes, st), "zero intermediate padding");
  // X = S B (S packed, mirrored on chip), then C = A X.
  if (int rc = run_contraction(AKind::SymmPacked, BKind::Dense, mode, structured_op(S, N), dense_op(b.ptr, b.ld), X,
                               ldx, N, N, N, st))
    return rc;
  return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, a.ld), dense_op(X, ldx), C, N, N, N, N, st);
}

// ---------------------------------------------------------------- structured right operand
extern "C" size_t smm_gen_x_struct_workspace_size(int M, int N, int mode) {
  (void)mode;
  if (M <= 0 || N <= 0) return 0;
  return round256(static_cast<size_t>(M) * round4(N) * sizeof(float));
}

namespace {
int gen_x_struct(const char* who, BKind bk, const float* A, const float* X, float* C, int M, int N, int mode, void* ws,
                 size_t ws_bytes, cudaStream_t st) {
  if (M < 0 || N < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!A || !X || !C) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  if (int rc = check_ws(who, ws, ws_bytes, pad_bytes(A, M, N))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a;
  if (int rc = stage_operand(A, M, N, cur, &a, st)) return rc;
  return run_contraction(AKind::Dense, bk, mode, dense_op(a.ptr, a.ld), structured_op(X, N), C, N, M, N, N, st);
}
}  // namespace

extern "C" int smm_gen_x_upper(const float* A, const float* U, float* C, int M, int N, int mode, void* ws,
                               size_t ws_bytes, void* stream) {
  return gen_x_struct("smm_gen_x_upper", BKind::UpperPacked, A, U, C, M, N, mode, ws, ws_bytes, as_stream(stream));
}

extern "C" int smm_gen_x_symm(const float* A, const float* S, float* C, int M, int N, int mode, void* ws,
                              size_t ws_bytes, void* stream) {
  return gen_x_struct("smm_gen_x_symm", BKind::SymmPacked, A, S, C, M, N, mode, ws, ws_bytes, as_stream(stream));
}

extern "C" int smm_symm_x_symm(const float* S1, const float* S2, float* C, int N, int mode, void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_symm_x_symm: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_x_symm: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!S1 || !S2 || !C) return set_error(SMM_ERR_INVALID, "smm_symm_x_symm: null pointer");
  return run_contraction(AKind::SymmPacked, BKind::SymmPacked, mode, structured_op(S1, N), structured_op(S2, N), C,
                         N, N, N, N, as_stream(stream));
}

// ---------------------------------------------------------------- timeout probe
namespace smm {
namespace {
__global__ void timeout_probe_kernel(uint32_t* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the bounded wait must give up on its own.
  const WaitCtx w{&abort_flag, status, limit_ns, kWaitProbe};
  mbar_wait(&bar, 0, w);
  __syncthreads();
}
}  // namespace
}  // namespace smm

extern "C" int smm_debug_timeout_probe(unsigned long long wait_limit, void* stream) {
  uint32_t* w = device_status_word();
  if (!w) return set_error(SMM_ERR_CUDA, "device status word unavailable");
  if (wait_limit == 0 || wait_limit > 10ull * 1000000000ull)
    return set_error(SMM_ERR_INVALID, "smm_debug_timeout_probe: limit must be in (0, 10 s]");
  cudaStream_t st = as_stream(stream);
  timeout_probe_kernel<<<1, 32, 0, st>>>(w, wait_limit);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "timeout probe launch");
  return smm_device_status(stream);
}

// Diagnostic: the next contraction launched from this thread records the
// state of its CTA (0,0) into `trace` (64 device words): TMEM base, k-block
// count, the first staged A/B words, shared-memory and instruction
// descriptors, and the first accumulator words read back.
extern "C" int smm_debug_trace_next(unsigned* trace) {
  g_trace = trace;
  return SMM_OK;
}

// ---------------------------------------------------------------- allocation-free sandwich
// Scratch of smm_symm_sandwich_noalloc: the S*B intermediate, plus padded
// copies of A and B when their rows are not 16-byte multiples.  A fixed
// 16 MiB that every GPU which loads this library holds until process exit.
// Host code must not use this name as an address (it is a host-side stand-in
// for the symbol); the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[size_t(16) << 20];

namespace smm {
namespace {
constexpr size_t kNoallocScratchBytes = sizeof(g_noalloc_scratch);

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  static void* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev & 63]) {
    void* p = nullptr;
    SMM_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(static sandwich scratch)");
    addr[dev & 63] = p;
  }
  *out = addr[dev & 63];
  return SMM_OK;
}
}  // namespace
}  // namespace smm

extern "C" int smm_symm_sandwich_noalloc(const float* A, const float* S, const float* B, float* C, int N, int mode,
                                         void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!A || !S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: null pointer");
  // Same scratch layout smm_symm_sandwich uses: X = S B with a 16-byte row
  // stride, then any padded operand copies.
  const size_t need = round256(static_cast<size_t>(N) * round4(N) * sizeof(float)) + pad_bytes(A, N, N) +
                      pad_bytes(B, N, N);
  if (need > kNoallocScratchBytes)
    return set_error(SMM_ERR_WORKSPACE,
                     "smm_symm_sandwich_noalloc: N = %d needs %zu bytes of scratch but the static scratch holds %zu "
                     "(N <= 2048 when N %% 4 == 0 and A, B are 16-byte aligned)",
                     N, need, kNoallocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return smm_symm_sandwich(A, S, B, C, N, mode, scratch, kNoallocScratchBytes, stream);
}
