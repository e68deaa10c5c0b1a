// libsmm host library: C ABI entry points for the tensor-core contractions
// on device buffers (dense GEMM, triangular / Toeplitz / symmetric operands
// on either side, the symmetric sandwich), the contraction driver
// (run_contraction: tile policy, TMA descriptors, launch), error/status
// plumbing, the timeout probe and the allocation-free sandwich.  Operand
// staging and expansion live in smm_stage.cu, the host-buffer pipeline in
// smm_host_pipe.cu.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "smm_contract.h"
#include "smm_host.h"
#include "smm_launch.cuh"

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

// Device address of g_smm_status on the current device (cached for device
// indices below 64; null for others or on failure).
uint32_t* device_status_word() {
  static uint32_t* addr[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_smm_status) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<uint32_t*>(p);
  }
  return addr[dev];
}

// Limit of every pipeline wait in the contraction kernels: SMM_WAIT_LIMIT_MS
// (a positive number of milliseconds; unset, 0 or unparsable keeps the
// 2000 ms default).  smm_debug_wait_limit_next sets a limit in nanoseconds
// for one launch.
unsigned long long wait_limit_ns() {
  static unsigned long long v = [] {
    const char* e = std::getenv("SMM_WAIT_LIMIT_MS");
    unsigned long long ms = e ? std::strtoull(e, nullptr, 10) : 0ull;
    if (ms == 0) ms = 2000ull;
    return ms * 1000000ull;
  }();
  return v;
}

// Teardown waits (for TMA copies and MMAs a CTA has already issued) get at
// least a second even when the pipeline limit is far shorter: a CTA must not
// exit while a bulk copy into its shared memory is still in flight.
constexpr unsigned long long kMinDrainNs = 1000000000ull;

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

// 2-D tensor map over a row-major matrix (rows x cols, leading dimension ld
// elements of fp32 or bf16), box of box_cols x box_rows elements.
int make_tmap(CUtensorMap* m, const void* base, int rows, int cols, int ld, int box_cols, int box_rows,
              CUtensorMapSwizzle swz, bool bf16 = false) {
  auto fn = encode_fn();
  if (!fn) return set_error(SMM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const size_t esz = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(SMM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %d x %d (ld %d)", int(r), rows, cols, ld);
  return SMM_OK;
}

// ---------------------------------------------------------------- launches
// CTA pairs (256-row tiles, tcgen05 cta_group::2) whenever there are at least
// two row tiles and the pair tiles fill about a wave of the 74 SM pairs.
// SMM_PAIR=0 forces single-CTA tiles, SMM_PAIR=1 pairs for every M > 128.
bool use_pairs(int M, int N) {
  const char* e = std::getenv("SMM_PAIR");
  if (e && e[0] == '0') return false;
  if (M <= kBM) return false;
  if (e && e[0] == '1') return true;
  const long long rp = (M + 2 * kBM - 1) / (2 * kBM);
  return rp * ((N + 127) / 128) >= 60;
}

// Output tile width: the widest tile that still yields about a wave of CTAs
// (of CTA pairs when pair is set).
int pick_bn(int M, int N, bool pair) {
  const char* e = std::getenv("SMM_TILE_N");
  if (e) {
    int v = std::atoi(e);
    if (v == 256 || v == 128 || (v == 64 && !pair)) return v;
  }
  // 128-wide pair tiles only when 256-wide ones would leave most pairs idle:
  // they measured far slower per FLOP (U B 4096 3xTF32: 146 against 198
  // TFLOP/s with 256-wide tiles, bf16 447 against 569), more than any wave
  // quantisation they save.
  if (pair) {
    const long long rp = (M + 2 * kBM - 1) / (2 * kBM);
    return (N > 128 && rp * ((N + 255) / 256) >= 60) ? 256 : 128;
  }
  const long long rt = (M + kBM - 1) / kBM;
  if (N > 128 && rt * ((N + 255) / 256) >= 120) return 256;
  if (N > 64 && rt * ((N + 127) / 128) >= 100) return 128;
  return 64;
}

// Split the K range of each 128 x 128 output tile over a cluster of two
// CTAs: dense (or dense upper-triangular) x dense products whose
// single-CTA tiles fill well under a wave (at most 74 tiles of 148 SMs) and
// whose longest K range gives each half at least 16 k-blocks (the heaviest
// row slab of a multi-GPU U B at 8 GPUs: 512 rows with K ~ 8000, where one
// 256 x 256 pair tile alone takes longer than the whole slab should).
// SMM_SPLITK=0 disables it, SMM_SPLITK=2 forces it for every such product
// without CTA pairs.
bool use_split(AKind ak, BKind bk, const Operand& a, const Operand& b, bool pair, int M, int N, int K) {
  if ((ak != AKind::Dense && ak != AKind::UpperDense) || bk != BKind::Dense || pair || a.lower || b.tri != 0)
    return false;
  const char* e = std::getenv("SMM_SPLITK");
  if (e && e[0] == '0') return false;
  if (e && e[0] == '2') return true;
  const long long tiles = static_cast<long long>((M + kBM - 1) / kBM) * ((N + 127) / 128);
  const int k_longest = ak == AKind::UpperDense ? K - a.row0 : K;
  return tiles <= 74 && k_longest >= 512;
}

// Diagnostic record target for the next contraction launch (set by
// smm_debug_trace_next, consumed by one launch).
thread_local uint32_t* g_trace = nullptr;
// Events recorded on the launch stream right before and after the next
// contraction kernel launched from this thread (smm_debug_time_next), and a
// pipeline wait limit for that launch (smm_debug_wait_limit_next).
thread_local cudaEvent_t g_ev_before = nullptr;
thread_local cudaEvent_t g_ev_after = nullptr;
thread_local unsigned long long g_wait_next = 0;

}  // namespace

bool valid_mode(int mode) { return mode == SMM_MODE_3XTF32 || mode == SMM_MODE_TF32 || mode == SMM_MODE_BF16; }

int check_packed(const char* who, int N) {
  if (N > kMaxPackedOrder)
    return set_error(SMM_ERR_INVALID, "%s: packed order N = %d exceeds %d", who, N, kMaxPackedOrder);
  return SMM_OK;
}

// Core contraction: C(M x N, ldc) = Aop(M x K) * B(K x N, ldb).
// Preconditions: B (and A when dense) 16-byte aligned with ld % 4 == 0.
int run_contraction(AKind ak, BKind bk, int mode, const Operand& a, const Operand& b, float* C, int ldc, int M,
                    int N, int K, cudaStream_t st, float* C_lo, __nv_bfloat16* C_bf16, int ldc_bf16,
                    TilePolicy policy) {
  const bool bf16 = (mode == SMM_MODE_BF16);
  const bool wide = policy == TilePolicy::WidePairs && M > kBM && N > 128;
  const bool pair = wide || use_pairs(M, N);
  const bool split = !wide && use_split(ak, bk, a, b, pair, M, N, K);
  const int bn = wide ? 256 : split ? 128 : pick_bn(M, N, pair);
  Maps m;
  const bool a_tma = (ak == AKind::Dense || ak == AKind::UpperDense);
  const bool b_tma = (bk == BKind::Dense);
  // fp32: A boxes 16 x 128 (64-byte swizzle), B boxes 32 x 16 (128-byte
  // swizzle, 32-byte atoms); bf16: A boxes 32 x 128, B boxes 64 x 32 (128-byte).
  const int a_box = bf16 ? 32 : 16;
  const int b_box_c = bf16 ? 64 : 32, b_box_r = bf16 ? 32 : 16;
  const CUtensorMapSwizzle b_swz = bf16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  if (b_tma) {
    const void* bp = bf16 ? static_cast<const void*>(b.bf16) : static_cast<const void*>(b.ptr);
    if (!bp) return set_error(SMM_ERR_INVALID, "internal: missing B operand plane");
    if (int rc = make_tmap(&m.b, bp, K, N, b.ld, b_box_c, b_box_r, b_swz, bf16)) return rc;
  }
  if (a_tma) {
    const void* ap = bf16 ? static_cast<const void*>(a.bf16) : static_cast<const void*>(a.ptr);
    if (!ap) return set_error(SMM_ERR_INVALID, "internal: missing A operand plane");
    if (int rc = make_tmap(&m.a, ap, M, K, a.ld, a_box, 128, CU_TENSOR_MAP_SWIZZLE_64B, bf16)) return rc;
  }
  UmmaParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.C_lo = C_lo;
  p.C_bf16 = C_bf16;
  p.ldc_bf16 = ldc_bf16;
  p.a_src = a.src;
  p.a_dim = a.dim;
  p.a_row0 = a.row0;
  if (a.tile_rows > 0) {
    if (ak != AKind::UpperDense || a.ntiles < 1 || a.ntiles > kMaxMappedTiles || !a.tile_row0 ||
        static_cast<long long>(a.ntiles) * a.tile_rows < M || a.tile_rows % (2 * kBM) != 0)
      return set_error(SMM_ERR_INVALID, "internal: bad row-tile map (%d tiles of %d rows for %d rows)", a.ntiles,
                       a.tile_rows, M);
    p.a_tile_rows = a.tile_rows;
    for (int i = 0; i < a.ntiles; ++i) p.a_tile_row0[i] = a.tile_row0[i];
  }
  p.a_lower = a.lower ? 1 : 0;
  p.b_tri = b.tri;
  p.b_src = b.src;
  p.b_dim = b.dim;
  p.row_tiles = pair ? (M + 2 * kBM - 1) / (2 * kBM) : (M + kBM - 1) / kBM;
  p.col_tiles = (N + bn - 1) / bn;
  // Rasterisation group (row tiles per group): 8 balances the re-reads of
  // A and B for TMA-fed operands (a wave of 74 pair tiles spans ~8 x 9
  // tiles); a Toeplitz A is built on chip from a generator that stays in L2,
  // so a group spans every row tile and each B column slab is read once.
  p.raster_group = ak == AKind::Toeplitz ? std::max(p.row_tiles, 1) : 8;
  p.status = device_status_word();
  p.wait_limit_ns = g_wait_next ? g_wait_next : wait_limit_ns();
  p.drain_limit_ns = std::max(p.wait_limit_ns, kMinDrainNs);
  p.trace = g_trace;
  g_trace = nullptr;
  g_wait_next = 0;
  cudaEvent_t ev_before = g_ev_before, ev_after = g_ev_after;
  g_ev_before = g_ev_after = nullptr;
  if (!p.status) return set_error(SMM_ERR_CUDA, "device status word unavailable");
  if (ev_before) SMM_CUDA_TRY(cudaEventRecord(ev_before, st), "record event before the contraction");
  // One-pass modes on TMA-fed operands with 256 x 256 pair tiles run
  // persistent: one CTA pair per SM pair walks the tiles with the
  // accumulator double-buffered in tensor memory (SMM_PERSIST=0 disables it).
  const char* pe = std::getenv("SMM_PERSIST");
  const bool persist = !(pe && pe[0] == '0') && !split && pair && bn == 256 && mode != SMM_MODE_3XTF32 &&
                       (ak == AKind::Dense || ak == AKind::UpperDense) && bk == BKind::Dense && !a.lower &&
                       b.tri == 0 && C_lo == nullptr && C_bf16 == nullptr;
  const int rc = split     ? launch_dense_split(ak, mode, m, p, st)
                 : persist ? launch_dense_persist(ak, mode, m, p, st)
                           : launch_kinds(ak, bk, bn, pair, mode, m, p, st);
  if (rc == SMM_OK && ev_after) SMM_CUDA_TRY(cudaEventRecord(ev_after, st), "record event after the contraction");
  return rc;
}

Operand dense_op(const float* ptr, const float* lo, int ld, const __nv_bfloat16* bf) {
  Operand o;
  o.ptr = ptr;
  o.lo = lo;
  o.ld = ld;
  o.bf16 = bf;
  return o;
}
Operand structured_op(const float* src, int dim, int row0) {
  Operand o;
  o.src = src;
  o.dim = dim;
  o.row0 = row0;
  return o;
}

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
    if (v & kDevErrBounds)
      return set_error(SMM_ERR_BOUNDS, "a bounds check caught an out-of-range read (status 0x%x); it was skipped", v);
  }
  return SMM_OK;
}

extern "C" size_t smm_gemm_workspace_size(int M, int N, int K, int mode) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return staged_bytes_bound(M, K, mode) + staged_bytes_bound(K, N, mode);
}

extern "C" int smm_gemm(const float* A, const float* B, float* C, int M, int N, int K, int mode, void* ws,
                        size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_gemm");
  if (M < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "smm_gemm: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_gemm: unknown mode %d", mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(SMM_ERR_INVALID, "smm_gemm: null pointer");
  cudaStream_t st = as_stream(stream);
  if (K == 0) return zero_output(C, M, N, st);
  const size_t need = staged_bytes(A, M, K, mode) + staged_bytes(B, K, N, mode);
  if (int rc = check_ws("smm_gemm", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a, b;
  if (int rc = stage_operand(A, M, K, mode, cur, &a, st)) return rc;
  if (int rc = stage_operand(B, K, N, mode, cur, &b, st)) return rc;
  return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, a.lo, a.ld, a.bf16), dense_op(b.ptr, b.lo, b.ld, b.bf16),
                         C, N, M, N, K, st);
}

extern "C" size_t smm_upper_left_workspace_size(int N, int ncols, int u_fmt, int mode) {
  if (N <= 0 || ncols <= 0) return 0;
  // + a staged copy of a dense U, or the expansion of a packed one
  return staged_bytes_bound(N, ncols, mode) + staged_bytes_bound(N, N, mode);
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
  SMM_RANGE("smm_upper_left_rows");
  if (int rc = check_slab("smm_upper_left", N, ncols, row0, nrows)) return rc;
  if (u_fmt == SMM_FMT_PACKED)
    if (int rc = check_packed("smm_upper_left", N)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_upper_left: unknown mode %d", mode);
  if (u_fmt != SMM_FMT_PACKED && u_fmt != SMM_FMT_DENSE)
    return set_error(SMM_ERR_INVALID, "smm_upper_left: unknown U format %d", u_fmt);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!U || !B || !C) return set_error(SMM_ERR_INVALID, "smm_upper_left: null pointer");
  cudaStream_t st = as_stream(stream);
  size_t need = staged_bytes(B, N, ncols, mode);
  if (u_fmt == SMM_FMT_DENSE) need += staged_bytes(U, N, N, mode);
  const bool expand =
      u_fmt == SMM_FMT_PACKED && expand_packed(ws, ws_bytes, need + expanded_bytes(nrows, N, mode));
  if (expand) need += expanded_bytes(nrows, N, mode);
  if (int rc = check_ws("smm_upper_left", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, mode, cur, &b, st)) return rc;
  if (u_fmt == SMM_FMT_DENSE) {
    Staged u;
    if (int rc = stage_operand(U, N, N, mode, cur, &u, st)) return rc;
    const size_t off = static_cast<size_t>(row0) * u.ld;
    Operand ua = dense_op(u.ptr ? u.ptr + off : nullptr, u.lo ? u.lo + off : nullptr, u.ld,
                          u.bf16 ? u.bf16 + off : nullptr);
    ua.dim = N;
    ua.row0 = row0;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ua, dense_op(b.ptr, b.lo, b.ld, b.bf16), C, ncols, nrows,
                           ncols, N, st);
  }
  if (expand) {
    Staged u;
    if (int rc = expand_operand(U, SMM_STRUCT_UPPER, N, row0, nrows, mode, cur, &u, st)) return rc;
    Operand ua = dense_op(u.ptr, nullptr, u.ld, u.bf16);
    ua.dim = N;
    ua.row0 = row0;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ua, dense_op(b.ptr, b.lo, b.ld, b.bf16), C, ncols, nrows,
                           ncols, N, st);
  }
  return run_contraction(AKind::UpperPacked, BKind::Dense, mode, structured_op(U, N, row0), dense_op(b.ptr, b.lo, b.ld, b.bf16),
                         C, ncols, nrows, ncols, N, st);
}

extern "C" int smm_upper_left(const float* U, int u_fmt, const float* B, float* C, int N, int ncols, int mode,
                              void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_upper_left");
  return smm_upper_left_rows(U, u_fmt, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

extern "C" size_t smm_toeplitz_left_workspace_size(int N, int ncols, int mode) {
  if (N <= 0 || ncols <= 0) return 0;
  return staged_bytes_bound(N, ncols, mode);
}

extern "C" int smm_toeplitz_left_rows(const float* g, const float* B, float* C, int N, int ncols, int row0,
                                      int nrows, int mode, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_toeplitz_left_rows");
  if (int rc = check_slab("smm_toeplitz_left", N, ncols, row0, nrows)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_toeplitz_left: unknown mode %d", mode);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!g || !B || !C) return set_error(SMM_ERR_INVALID, "smm_toeplitz_left: null pointer");
  cudaStream_t st = as_stream(stream);
  if (int rc = check_ws("smm_toeplitz_left", ws, ws_bytes, staged_bytes(B, N, ncols, mode))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, mode, cur, &b, st)) return rc;
  return run_contraction(AKind::Toeplitz, BKind::Dense, mode, structured_op(g, N, row0), dense_op(b.ptr, b.lo, b.ld, b.bf16), C,
                         ncols, nrows, ncols, N, st);
}

extern "C" int smm_toeplitz_left(const float* g, const float* B, float* C, int N, int ncols, int mode, void* ws,
                                 size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_toeplitz_left");
  return smm_toeplitz_left_rows(g, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

extern "C" size_t smm_symm_left_workspace_size(int N, int ncols, int mode) {
  if (N <= 0 || ncols <= 0) return 0;
  return staged_bytes_bound(N, ncols, mode) + expanded_bytes(N, N, mode);
}

extern "C" int smm_symm_left_rows(const float* S, const float* B, float* C, int N, int ncols, int row0, int nrows,
                                  int mode, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_symm_left_rows");
  if (int rc = check_slab("smm_symm_left", N, ncols, row0, nrows)) return rc;
  if (int rc = check_packed("smm_symm_left", N)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_left: unknown mode %d", mode);
  if (nrows == 0 || ncols == 0) return SMM_OK;
  if (!S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_left: null pointer");
  cudaStream_t st = as_stream(stream);
  const size_t need_b = staged_bytes(B, N, ncols, mode);
  const bool expand = expand_packed(ws, ws_bytes, need_b + expanded_bytes(nrows, N, mode));
  if (int rc = check_ws("smm_symm_left", ws, ws_bytes, need_b + (expand ? expanded_bytes(nrows, N, mode) : 0)))
    return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, mode, cur, &b, st)) return rc;
  if (expand) {
    Staged s;
    if (int rc = expand_operand(S, SMM_STRUCT_SYMM, N, row0, nrows, mode, cur, &s, st)) return rc;
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(s.ptr, nullptr, s.ld, s.bf16),
                           dense_op(b.ptr, b.lo, b.ld, b.bf16), C, ncols, nrows, ncols, N, st);
  }
  return run_contraction(AKind::SymmPacked, BKind::Dense, mode, structured_op(S, N, row0), dense_op(b.ptr, b.lo, b.ld, b.bf16),
                         C, ncols, nrows, ncols, N, st);
}

extern "C" int smm_symm_left(const float* S, const float* B, float* C, int N, int ncols, int mode, void* ws,
                             size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_symm_left");
  return smm_symm_left_rows(S, B, C, N, ncols, 0, N, mode, ws, ws_bytes, stream);
}

namespace {
// Workspace of the sandwich: X = S B (16-byte row stride) and, in bf16 mode,
// its bf16 copy (written by the first product's epilogue), the dense
// expansion of S when there is room for it, then the staged A and B.
size_t sandwich_x_bytes(int N, int mode) {
  if (mode == SMM_MODE_BF16) return plane_bytes(N, N) + bf16_plane_bytes(N, N);
  return plane_bytes(N, N);
}
// Without the expansion of S.
size_t sandwich_need(const float* A, const float* B, int N, int mode) {
  return sandwich_x_bytes(N, mode) + staged_bytes(A, N, N, mode) + staged_bytes(B, N, N, mode);
}
}  // namespace

extern "C" size_t smm_symm_sandwich_workspace_size(int N, int mode) {
  if (N <= 0) return 0;
  return sandwich_x_bytes(N, mode) + expanded_bytes(N, N, mode) + 2 * staged_bytes_bound(N, N, mode);
}

extern "C" int smm_symm_sandwich(const float* A, const float* S, const float* B, float* C, int N, int mode,
                                 void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_symm_sandwich");
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!A || !S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich: null pointer");
  if (int rc = check_packed("smm_symm_sandwich", N)) return rc;
  cudaStream_t st = as_stream(stream);
  const bool bf = (mode == SMM_MODE_BF16);
  const size_t need = sandwich_need(A, B, N, mode);
  const bool expand = expand_packed(ws, ws_bytes, need + expanded_bytes(N, N, mode));
  if (int rc = check_ws("smm_symm_sandwich", ws, ws_bytes, need + (expand ? expanded_bytes(N, N, mode) : 0)))
    return rc;
  const int ldx = round4(N);
  const int ldx_bf = round8(N);
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* X = reinterpret_cast<float*>(cur);
  cur += plane_bytes(N, N);
  float* X_lo = nullptr;
  __nv_bfloat16* X_bf = nullptr;
  if (bf) {
    X_bf = reinterpret_cast<__nv_bfloat16*>(cur);
    cur += bf16_plane_bytes(N, N);
    // the bf16 row padding must read as zeros (never multiplied, but keep it defined)
    if (ldx_bf != N) SMM_CUDA_TRY(cudaMemsetAsync(X_bf, 0, bf16_plane_bytes(N, N), st), "zero bf16 intermediate");
  }
  Staged s_ex{};
  if (expand)
    if (int rc = expand_operand(S, SMM_STRUCT_SYMM, N, 0, N, mode, cur, &s_ex, st)) return rc;
  Staged a, b;
  if (int rc = stage_operand(A, N, N, mode, cur, &a, st)) return rc;
  if (int rc = stage_operand(B, N, N, mode, cur, &b, st)) return rc;
  // X = S B (S expanded, or packed and mirrored on chip; in bf16 mode the
  // epilogue writes only X's bf16 copy, the second product's operand), then
  // C = A X.
  const Operand s_op = expand ? dense_op(s_ex.ptr, nullptr, s_ex.ld, s_ex.bf16) : structured_op(S, N);
  if (int rc = run_contraction(expand ? AKind::Dense : AKind::SymmPacked, BKind::Dense, mode, s_op,
                               dense_op(b.ptr, b.lo, b.ld, b.bf16), bf ? nullptr : X, ldx, N, N, N, st, X_lo, X_bf,
                               ldx_bf))
    return rc;
  return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, a.lo, a.ld, a.bf16),
                         dense_op(X, X_lo, bf ? ldx_bf : ldx, X_bf), C, N, N, N, N, st);
}

// ---------------------------------------------------------------- structured right operand
extern "C" size_t smm_gen_x_struct_workspace_size(int M, int N, int mode) {
  if (M <= 0 || N <= 0) return 0;
  return staged_bytes_bound(M, N, mode) + expanded_bytes(N, N, mode);
}

namespace {
int gen_x_struct(const char* who, BKind bk, const float* A, const float* X, float* C, int M, int N, int mode, void* ws,
                 size_t ws_bytes, cudaStream_t st) {
  if (M < 0 || N < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!A || !X || !C) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  if (int rc = check_packed(who, N)) return rc;
  // The packed right operand is expanded into a dense copy (read by TMA, its
  // K range clipped per column tile when triangular) when the workspace has
  // room for it, else built on chip by the transform warps.
  const size_t need_a = staged_bytes(A, M, N, mode);
  const bool expand = expand_packed(ws, ws_bytes, need_a + expanded_bytes(N, N, mode));
  if (int rc = check_ws(who, ws, ws_bytes, need_a + (expand ? expanded_bytes(N, N, mode) : 0))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a;
  if (int rc = stage_operand(A, M, N, mode, cur, &a, st)) return rc;
  if (expand) {
    const int sf = bk == BKind::UpperPacked ? SMM_STRUCT_UPPER : (bk == BKind::LowerPacked ? SMM_STRUCT_LOWER : SMM_STRUCT_SYMM);
    Staged x;
    if (int rc = expand_operand(X, sf, N, 0, N, mode, cur, &x, st)) return rc;
    Operand xb = dense_op(x.ptr, nullptr, x.ld, x.bf16);
    xb.tri = sf == SMM_STRUCT_UPPER ? 1 : (sf == SMM_STRUCT_LOWER ? 2 : 0);
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, a.lo, a.ld, a.bf16), xb, C, N, M, N, N, st);
  }
  return run_contraction(AKind::Dense, bk, mode, dense_op(a.ptr, a.lo, a.ld, a.bf16), structured_op(X, N), C, N, M, N, N, st);
}
}  // namespace

extern "C" int smm_gen_x_upper(const float* A, const float* U, float* C, int M, int N, int mode, void* ws,
                               size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_gen_x_upper");
  return gen_x_struct("smm_gen_x_upper", BKind::UpperPacked, A, U, C, M, N, mode, ws, ws_bytes, as_stream(stream));
}

extern "C" int smm_gen_x_symm(const float* A, const float* S, float* C, int M, int N, int mode, void* ws,
                              size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_gen_x_symm");
  return gen_x_struct("smm_gen_x_symm", BKind::SymmPacked, A, S, C, M, N, mode, ws, ws_bytes, as_stream(stream));
}

extern "C" int smm_gen_x_lower(const float* A, const float* Lp, float* C, int M, int N, int mode, void* ws,
                               size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_gen_x_lower");
  return gen_x_struct("smm_gen_x_lower", BKind::LowerPacked, A, Lp, C, M, N, mode, ws, ws_bytes, as_stream(stream));
}

extern "C" size_t smm_gen_x_toeplitz_workspace_size(int M, int N, int K, int mode) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return staged_bytes_bound(M, K, mode) + toeplitz_expanded_bytes(K, N, mode);
}

extern "C" int smm_gen_x_toeplitz(const float* A, const float* g, float* C, int M, int N, int K, int mode, void* ws,
                                  size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_gen_x_toeplitz");
  if (M < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "smm_gen_x_toeplitz: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_gen_x_toeplitz: unknown mode %d", mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!C || (K > 0 && (!A || !g))) return set_error(SMM_ERR_INVALID, "smm_gen_x_toeplitz: null pointer");
  cudaStream_t st = as_stream(stream);
  if (K == 0) return zero_output(C, M, N, st);
  // The Toeplitz right operand is expanded into a dense K x N copy (TMA-fed)
  // when the workspace has room for it, else built on chip from the
  // generator by the transform warps.
  const size_t need_a = staged_bytes(A, M, K, mode);
  const bool expand = expand_packed(ws, ws_bytes, need_a + toeplitz_expanded_bytes(K, N, mode));
  if (int rc = check_ws("smm_gen_x_toeplitz", ws, ws_bytes, need_a + (expand ? toeplitz_expanded_bytes(K, N, mode) : 0)))
    return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a;
  if (int rc = stage_operand(A, M, K, mode, cur, &a, st)) return rc;
  const Operand ao = dense_op(a.ptr, a.lo, a.ld, a.bf16);
  if (expand) {
    Staged t;
    if (int rc = expand_toeplitz(g, K, N, mode, cur, &t, st)) return rc;
    return run_contraction(AKind::Dense, BKind::Dense, mode, ao, dense_op(t.ptr, nullptr, t.ld, t.bf16), C, N, M, N,
                           K, st);
  }
  return run_contraction(AKind::Dense, BKind::Toeplitz, mode, ao, structured_op(g, K), C, N, M, N, K, st);
}

extern "C" int smm_symm_x_symm(const float* S1, const float* S2, float* C, int N, int mode, void* stream) {
  SMM_RANGE("smm_symm_x_symm");
  return smm_symm_x_symm_ws(S1, S2, C, N, mode, nullptr, 0, stream);
}

namespace {
// Product of two packed operands of order N: both expanded into dense copies
// in the workspace when it has room for them (TMA-fed; a lower-triangular
// left copy clips each row tile's K range from above, a lower-triangular
// right copy each column tile's from below), else both built on chip.
int packed_x_packed(const char* who, AKind ak, BKind bk, int sf, const float* X1, const float* X2, float* C, int N,
                    int mode, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (N == 0) return SMM_OK;
  if (!X1 || !X2 || !C) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  if (int rc = check_packed(who, N)) return rc;
  if (!expand_packed(ws, ws_bytes, 2 * expanded_bytes(N, N, mode)))
    return run_contraction(ak, bk, mode, structured_op(X1, N), structured_op(X2, N), C, N, N, N, N, st);
  if (int rc = check_ws(who, ws, ws_bytes, 2 * expanded_bytes(N, N, mode))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a, b;
  if (int rc = expand_operand(X1, sf, N, 0, N, mode, cur, &a, st)) return rc;
  if (int rc = expand_operand(X2, sf, N, 0, N, mode, cur, &b, st)) return rc;
  Operand ao = dense_op(a.ptr, nullptr, a.ld, a.bf16), bo = dense_op(b.ptr, nullptr, b.ld, b.bf16);
  ao.lower = sf == SMM_STRUCT_LOWER;
  bo.tri = sf == SMM_STRUCT_LOWER ? 2 : 0;
  return run_contraction(AKind::Dense, BKind::Dense, mode, ao, bo, C, N, N, N, N, st);
}
}  // namespace

extern "C" size_t smm_symm_x_symm_workspace_size(int N, int mode) {
  return N <= 0 ? 0 : 2 * expanded_bytes(N, N, mode);
}

extern "C" int smm_symm_x_symm_ws(const float* S1, const float* S2, float* C, int N, int mode, void* ws,
                                  size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_symm_x_symm_ws");
  return packed_x_packed("smm_symm_x_symm", AKind::SymmPacked, BKind::SymmPacked, SMM_STRUCT_SYMM, S1, S2, C, N,
                         mode, ws, ws_bytes, as_stream(stream));
}

// ---------------------------------------------------------------- lower-triangular operands
extern "C" size_t smm_lower_left_workspace_size(int N, int ncols, int mode) {
  if (N <= 0 || ncols <= 0) return 0;
  return staged_bytes_bound(N, ncols, mode) + expanded_bytes(N, N, mode);
}

extern "C" int smm_lower_left(const float* Lp, const float* B, float* C, int N, int ncols, int mode, void* ws,
                              size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_lower_left");
  if (N < 0 || ncols < 0) return set_error(SMM_ERR_INVALID, "smm_lower_left: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_lower_left: unknown mode %d", mode);
  if (N == 0 || ncols == 0) return SMM_OK;
  if (!Lp || !B || !C) return set_error(SMM_ERR_INVALID, "smm_lower_left: null pointer");
  if (int rc = check_packed("smm_lower_left", N)) return rc;
  cudaStream_t st = as_stream(stream);
  const size_t need_b = staged_bytes(B, N, ncols, mode);
  const bool expand = expand_packed(ws, ws_bytes, need_b + expanded_bytes(N, N, mode));
  if (int rc = check_ws("smm_lower_left", ws, ws_bytes, need_b + (expand ? expanded_bytes(N, N, mode) : 0)))
    return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged b;
  if (int rc = stage_operand(B, N, ncols, mode, cur, &b, st)) return rc;
  if (expand) {
    Staged l;
    if (int rc = expand_operand(Lp, SMM_STRUCT_LOWER, N, 0, N, mode, cur, &l, st)) return rc;
    Operand la = dense_op(l.ptr, nullptr, l.ld, l.bf16);
    la.lower = true;
    return run_contraction(AKind::Dense, BKind::Dense, mode, la, dense_op(b.ptr, b.lo, b.ld, b.bf16), C, ncols, N,
                           ncols, N, st);
  }
  return run_contraction(AKind::LowerPacked, BKind::Dense, mode, structured_op(Lp, N), dense_op(b.ptr, b.lo, b.ld, b.bf16),
                         C, ncols, N, ncols, N, st);
}

extern "C" int smm_lower_x_lower(const float* L1, const float* L2, float* C, int N, int mode, void* stream) {
  SMM_RANGE("smm_lower_x_lower");
  return smm_lower_x_lower_ws(L1, L2, C, N, mode, nullptr, 0, stream);
}

extern "C" size_t smm_lower_x_lower_workspace_size(int N, int mode) {
  return N <= 0 ? 0 : 2 * expanded_bytes(N, N, mode);
}

extern "C" int smm_lower_x_lower_ws(const float* L1, const float* L2, float* C, int N, int mode, void* ws,
                                    size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_lower_x_lower_ws");
  return packed_x_packed("smm_lower_x_lower", AKind::LowerPacked, BKind::LowerPacked, SMM_STRUCT_LOWER, L1, L2, C, N,
                         mode, ws, ws_bytes, as_stream(stream));
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
  SMM_RANGE("smm_debug_timeout_probe");
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
  SMM_RANGE("smm_debug_trace_next");
  g_trace = trace;
  return SMM_OK;
}

// Measurement: the next contraction kernel launched from this thread is
// bracketed by cudaEventRecord(before) and cudaEventRecord(after) on its
// stream, so the caller can time that kernel alone (staging and expansion
// kernels of the same call fall outside the pair).  Either may be NULL.
extern "C" int smm_debug_time_next(void* event_before, void* event_after) {
  g_ev_before = static_cast<cudaEvent_t>(event_before);
  g_ev_after = static_cast<cudaEvent_t>(event_after);
  return SMM_OK;
}

// Failure-path test: the next contraction kernel launched from this thread
// gives every pipeline wait `wait_limit_ns` nanoseconds instead of the
// default (teardown waits keep at least a second).  0 restores the default.
extern "C" int smm_debug_wait_limit_next(unsigned long long wait_limit_ns) {
  if (wait_limit_ns > 10ull * 1000000000ull)
    return set_error(SMM_ERR_INVALID, "smm_debug_wait_limit_next: limit must be at most 10 s");
  g_wait_next = wait_limit_ns;
  return SMM_OK;
}

// ---------------------------------------------------------------- allocation-free sandwich
// Scratch of smm_symm_sandwich_noalloc: the S*B intermediate, plus padded
// copies of A and B when their rows are not 16-byte multiples, or the bf16
// copies in bf16 mode.  A fixed 16 MiB that every GPU which loads this library
// holds until process exit.
// Host code must not use this name as an address (it is a host-side stand-in
// for the symbol); the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[size_t(16) << 20];

namespace smm {
namespace {
constexpr size_t kNoallocScratchBytes = sizeof(g_noalloc_scratch);

constexpr int kMaxCachedDevices = 64;

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  static void* addr[kMaxCachedDevices] = {};
  static std::mutex mu;
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxCachedDevices)
    return set_error(SMM_ERR_UNSUPPORTED, "smm_symm_sandwich_noalloc: device index %d (at most %d devices)", dev,
                     kMaxCachedDevices);
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    SMM_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(static sandwich scratch)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return SMM_OK;
}
}  // namespace
}  // namespace smm

extern "C" int smm_symm_sandwich_noalloc(const float* A, const float* S, const float* B, float* C, int N, int mode,
                                         void* stream) {
  SMM_RANGE("smm_symm_sandwich_noalloc");
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: negative shape");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!A || !S || !B || !C) return set_error(SMM_ERR_INVALID, "smm_symm_sandwich_noalloc: null pointer");
  // Same scratch layout smm_symm_sandwich uses.
  const size_t need = sandwich_need(A, B, N, mode);
  if (need > kNoallocScratchBytes)
    return set_error(SMM_ERR_WORKSPACE,
                     "smm_symm_sandwich_noalloc: N = %d needs %zu bytes of scratch but the static scratch holds %zu "
                     "(fp32 modes: N <= 2048 with N %% 4 == 0 and 16-byte-aligned A, B, else N <= 1180; "
                     "bf16: N <= 1294)",
                     N, need, kNoallocScratchBytes);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return smm_symm_sandwich(A, S, B, C, N, mode, scratch, kNoallocScratchBytes, stream);
}
