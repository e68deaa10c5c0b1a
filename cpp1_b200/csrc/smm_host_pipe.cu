// Host-buffer contractions (smm_*_host): C = L B with every operand in host
// memory, the left operand(s) copied once and B streamed in column chunks
// whose copies overlap the products.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "smm_contract.h"

// C = L B with L, B and C in host memory (pinned for overlap; pageable works,
// synchronously): the drop-in for callers of the reference's CPU kernels,
// which take host arrays.  The left operand(s) cross PCIe once and are
// prepared on the device (staged, or a packed operand expanded) on a stream
// of their own; B streams through in column chunks, chunk j in buffer region
// j % 2.  The region's chunk stream orders chunk j's 2-D copy-in (which does
// not wait for the left operand, so B's first chunks cross PCIe while the
// left operand is being expanded) and its product (which does); the 2-D
// copy-out into C's columns runs on the region's copy-out stream once the
// product is done.  So chunk j+2's copy-in waits only for chunk j's product
// (its B buffer), not for chunk j's copy-out: PCIe is full duplex, and the
// host-to-device copies keep flowing while results drain.  Chunk j+2's
// product waits for chunk j's copy-out (its C buffer).
namespace smm {
namespace {

enum class HostLeft { Gemm, Upper, Symm, Toeplitz, Sandwich };

struct HostStreams {
  cudaStream_t st[2] = {nullptr, nullptr};  // chunks of region k: copy-in, product
  cudaStream_t so[2] = {nullptr, nullptr};  // chunks of region k: copy-out
  cudaStream_t sl = nullptr;                // the left operand(s): copy in and prepare
  cudaEvent_t left_ready = nullptr;
  cudaEvent_t prod_done[2] = {nullptr, nullptr};  // region k's latest product
  cudaEvent_t out_done[2] = {nullptr, nullptr};   // region k's latest copy-out
  bool init = false;
};

// After chunk product(s) on st: the copy-out on the region's copy-out stream,
// then record its completion (the region's next product waits for it).
int chunk_copy_out(HostStreams* hs, int k, void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                   size_t height) {
  SMM_CUDA_TRY(cudaEventRecord(hs->prod_done[k], hs->st[k]), "event record");
  SMM_CUDA_TRY(cudaStreamWaitEvent(hs->so[k], hs->prod_done[k], 0), "wait for the chunk product");
  if (height == 1)
    SMM_CUDA_TRY(cudaMemcpyAsync(dst, src, width, cudaMemcpyDeviceToHost, hs->so[k]), "copy C chunk");
  else
    SMM_CUDA_TRY(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDeviceToHost, hs->so[k]),
                 "copy C chunk");
  SMM_CUDA_TRY(cudaEventRecord(hs->out_done[k], hs->so[k]), "event record");
  return SMM_OK;
}

// The caller's view at the end of a host-buffer product: every stream drained.
int drain_host_streams(HostStreams* hs) {
  for (int k = 0; k < 2; ++k) {
    SMM_CUDA_TRY(cudaStreamSynchronize(hs->st[k]), "stream sync");
    SMM_CUDA_TRY(cudaStreamSynchronize(hs->so[k]), "stream sync");
  }
  SMM_CUDA_TRY(cudaStreamSynchronize(hs->sl), "stream sync");
  return SMM_OK;
}

int host_streams(HostStreams** out) {
  static HostStreams per_dev[64];
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(SMM_ERR_UNSUPPORTED, "host-buffer entry points: device index %d >= 64", dev);
  HostStreams& h = per_dev[dev];
  // first call on this device: create its streams (once, even when several
  // host threads make their first call together)
  static std::mutex init_mu;
  std::lock_guard<std::mutex> lock(init_mu);
  if (!h.init) {
    for (auto& s : h.st) SMM_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
    for (auto& s : h.so) SMM_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream create");
    SMM_CUDA_TRY(cudaStreamCreateWithFlags(&h.sl, cudaStreamNonBlocking), "stream create");
    SMM_CUDA_TRY(cudaEventCreateWithFlags(&h.left_ready, cudaEventDisableTiming), "event create");
    for (int k = 0; k < 2; ++k) {
      SMM_CUDA_TRY(cudaEventCreateWithFlags(&h.prod_done[k], cudaEventDisableTiming), "event create");
      SMM_CUDA_TRY(cudaEventCreateWithFlags(&h.out_done[k], cudaEventDisableTiming), "event create");
    }
    h.init = true;
  }
  *out = &h;
  return SMM_OK;
}

// Columns of B per chunk: about an eighth of N in multiples of 256, at least
// 1024 (narrower products lose too much to partial waves), at most N.
int host_chunk_cols(int N) { return std::min(N, std::max(1024, (N / 8 + 255) / 256 * 256)); }

// Shapes: C is M x N, L is M x K; the sandwich has M = K = N.
struct HostShape {
  HostLeft kind;
  int M, N, K, mode;
};

size_t left_raw_bytes(const HostShape& h) {
  switch (h.kind) {
    case HostLeft::Gemm: return round256(static_cast<size_t>(h.M) * h.K * 4);
    case HostLeft::Upper:
    case HostLeft::Symm: return round256(static_cast<size_t>(h.K) * (h.K + 1) / 2 * 4);
    case HostLeft::Toeplitz: return round256((2 * static_cast<size_t>(h.K) - 1) * 4);
    default: return round256(static_cast<size_t>(h.N) * h.N * 4) + round256(static_cast<size_t>(h.N) * (h.N + 1) / 2 * 4);
  }
}
size_t left_prep_bytes(const HostShape& h) {
  switch (h.kind) {
    case HostLeft::Gemm: return staged_bytes_bound(h.M, h.K, h.mode);
    case HostLeft::Upper:
    case HostLeft::Symm: return expanded_bytes(h.K, h.K, h.mode);
    case HostLeft::Toeplitz: return 0;
    default: return staged_bytes_bound(h.N, h.N, h.mode) + expanded_bytes(h.N, h.N, h.mode);
  }
}
// One stream's chunk buffers: raw B chunk, its staged copy, the sandwich's X
// chunk (+ bf16 copy), the C chunk.
size_t chunk_bytes(const HostShape& h) {
  const int w = host_chunk_cols(h.N);
  size_t b = round256(static_cast<size_t>(h.K) * w * 4) + staged_bytes_bound(h.K, w, h.mode) +
             round256(static_cast<size_t>(h.M) * w * 4);
  if (h.kind == HostLeft::Sandwich) b += plane_bytes(h.N, w) + bf16_plane_bytes(h.N, w);
  return b;
}
size_t host_ws_bytes(const HostShape& h) {
  if (h.M <= 0 || h.N <= 0 || h.K <= 0) return 0;
  return left_raw_bytes(h) + left_prep_bytes(h) + 2 * chunk_bytes(h);
}

int host_product(const char* who, const HostShape& h, const float* L1, const float* L2, const float* B, float* C,
                 void* dev_ws, size_t ws_bytes) {
  const int M = h.M, N = h.N, K = h.K, mode = h.mode;
  if (M < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (M == 0 || N == 0) return SMM_OK;
  if (!L1 || !B || !C || (h.kind == HostLeft::Sandwich && !L2)) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  if (h.kind == HostLeft::Upper || h.kind == HostLeft::Symm || h.kind == HostLeft::Sandwich)
    if (int rc = check_packed(who, K)) return rc;
  if (K == 0) {  // an empty inner dimension: C = 0
    std::memset(C, 0, sizeof(float) * static_cast<size_t>(M) * N);
    return SMM_OK;
  }
  if (int rc = check_ws(who, dev_ws, ws_bytes, host_ws_bytes(h))) return rc;
  HostStreams* hs = nullptr;
  if (int rc = host_streams(&hs)) return rc;
  cudaStream_t s0 = hs->sl;  // the left operand's stream

  // ---- left operand(s): copy in once, prepare on their own stream
  uint8_t* cur = static_cast<uint8_t*>(dev_ws);
  Operand left, amat;  // amat: the sandwich's A
  if (h.kind == HostLeft::Gemm || h.kind == HostLeft::Sandwich) {
    float* a = reinterpret_cast<float*>(cur);
    const size_t ab = static_cast<size_t>(M) * K * 4;
    cur += round256(ab);
    SMM_CUDA_TRY(cudaMemcpyAsync(a, L1, ab, cudaMemcpyHostToDevice, s0), "copy A");
    Staged st;
    if (int rc = stage_operand(a, M, K, mode, cur, &st, s0)) return rc;
    amat = dense_op(st.ptr, st.lo, st.ld, st.bf16);
    left = amat;
  }
  if (h.kind != HostLeft::Gemm) {
    const float* src = h.kind == HostLeft::Sandwich ? L2 : L1;
    const size_t len = h.kind == HostLeft::Toeplitz ? 2 * static_cast<size_t>(K) - 1 : static_cast<size_t>(K) * (K + 1) / 2;
    float* p = reinterpret_cast<float*>(cur);
    cur += round256(len * 4);
    SMM_CUDA_TRY(cudaMemcpyAsync(p, src, len * 4, cudaMemcpyHostToDevice, s0), "copy structured operand");
    if (h.kind == HostLeft::Toeplitz) {
      left = structured_op(p, K);
    } else {
      const int sf = h.kind == HostLeft::Upper ? SMM_STRUCT_UPPER : SMM_STRUCT_SYMM;
      Staged ex;
      if (int rc = expand_operand(p, sf, K, 0, K, mode, cur, &ex, s0)) return rc;
      left = dense_op(ex.ptr, nullptr, ex.ld, ex.bf16);
      left.dim = K;
    }
  }
  const AKind lk = h.kind == HostLeft::Toeplitz ? AKind::Toeplitz
                   : h.kind == HostLeft::Upper  ? AKind::UpperDense
                                                : AKind::Dense;
  SMM_CUDA_TRY(cudaEventRecord(hs->left_ready, s0), "event record");

  // ---- B in column chunks, alternating streams
  const int w = host_chunk_cols(N);
  uint8_t* region[2] = {cur, cur + chunk_bytes(h)};
  int c = 0;
  for (int c0 = 0; c0 < N; c0 += w, ++c) {
    const int k = c & 1;
    const int wc = std::min(w, N - c0);
    cudaStream_t st = hs->st[k];
    uint8_t* r = region[k];
    float* braw = reinterpret_cast<float*>(r);
    r += round256(static_cast<size_t>(K) * w * 4);
    uint8_t* stage_cur = r;
    r += staged_bytes_bound(K, w, mode);
    float* xch = nullptr;
    __nv_bfloat16* xbf = nullptr;
    if (h.kind == HostLeft::Sandwich) {
      xch = reinterpret_cast<float*>(r);
      r += plane_bytes(N, w);
      xbf = reinterpret_cast<__nv_bfloat16*>(r);
      r += bf16_plane_bytes(N, w);
    }
    float* cch = reinterpret_cast<float*>(r);
    SMM_CUDA_TRY(cudaMemcpy2DAsync(braw, static_cast<size_t>(wc) * 4, B + c0, static_cast<size_t>(N) * 4,
                                   static_cast<size_t>(wc) * 4, K, cudaMemcpyHostToDevice, st),
                 "copy B chunk");
    Staged bs;
    if (int rc = stage_operand(braw, K, wc, mode, stage_cur, &bs, st)) return rc;
    const Operand bop = dense_op(bs.ptr, bs.lo, bs.ld, bs.bf16);
    if (c < 2) SMM_CUDA_TRY(cudaStreamWaitEvent(st, hs->left_ready, 0), "wait for the left operand");
    if (c >= 2) SMM_CUDA_TRY(cudaStreamWaitEvent(st, hs->out_done[k], 0), "wait for the C buffer");
    if (h.kind == HostLeft::Sandwich) {
      // X_j = S B_j (its bf16 copy too in bf16 mode), then C_j = A X_j
      const int ldx = round4(wc), ldx_bf = round8(wc);
      const bool bf = mode == SMM_MODE_BF16;
      if (bf && ldx_bf != wc)
        SMM_CUDA_TRY(cudaMemsetAsync(xbf, 0, bf16_plane_bytes(N, wc), st), "zero bf16 intermediate");
      if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, left, bop, xch, ldx, N, wc, N, st, nullptr,
                                   bf ? xbf : nullptr, ldx_bf))
        return rc;
      if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, amat,
                                   dense_op(xch, nullptr, bf ? ldx_bf : ldx, bf ? xbf : nullptr), cch, wc, N, wc, N,
                                   st))
        return rc;
    } else {
      if (int rc = run_contraction(lk, BKind::Dense, mode, left, bop, cch, wc, M, wc, K, st)) return rc;
    }
    if (int rc = chunk_copy_out(hs, k, C + c0, static_cast<size_t>(N) * 4, cch, static_cast<size_t>(wc) * 4,
                                static_cast<size_t>(wc) * 4, M))
      return rc;
  }
  if (int rc = drain_host_streams(hs)) return rc;
  return smm_device_status(s0);
}

// ---------------------------------------------------------------- right-side structured operand
// C (M x N) = A (M x K) X (K x N) with X structured (packed upper or
// symmetric, K = N; or a K + N - 1 Toeplitz generator): the orientation of
// the reference's CPU kernels (upper_triag_matmul.cpp:41-137 A*U,
// symmetric_matmul.cpp:84-211 A*S, toeplitz_matmul2.cpp:44-144 A*T).  X
// crosses PCIe once and is expanded into a dense copy on its own stream; A
// goes through in row chunks (contiguous in host memory) alternating between
// the two buffer regions, with the same streams and ordering as the column
// chunks of B above.
enum class HostRight { Upper, Symm, Toeplitz };

int host_row_chunk(int M) { return std::min(M, std::max(1024, (M / 8 + 255) / 256 * 256)); }

size_t right_raw_bytes(HostRight k, int N, int K) {
  return k == HostRight::Toeplitz ? round256((static_cast<size_t>(K) + N - 1) * 4)
                                  : round256(static_cast<size_t>(K) * (K + 1) / 2 * 4);
}
size_t right_chunk_bytes(int M, int N, int K, int mode) {
  const int h = host_row_chunk(M);
  return round256(static_cast<size_t>(h) * K * 4) + staged_bytes_bound(h, K, mode) +
         round256(static_cast<size_t>(h) * N * 4);
}
size_t host_right_ws(HostRight k, int M, int N, int K, int mode) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return right_raw_bytes(k, N, K) + toeplitz_expanded_bytes(K, N, mode) + 2 * right_chunk_bytes(M, N, K, mode);
}

int host_right_product(const char* who, HostRight kind, int M, int N, int K, int mode, const float* A,
                       const float* X, float* C, void* dev_ws, size_t ws_bytes) {
  if (M < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "%s: negative shape", who);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (kind != HostRight::Toeplitz && K != N) return set_error(SMM_ERR_INVALID, "%s: K must equal N", who);
  if (M == 0 || N == 0) return SMM_OK;
  if (!A || !X || !C) return set_error(SMM_ERR_INVALID, "%s: null pointer", who);
  if (kind != HostRight::Toeplitz)
    if (int rc = check_packed(who, N)) return rc;
  if (K == 0) {
    std::memset(C, 0, sizeof(float) * static_cast<size_t>(M) * N);
    return SMM_OK;
  }
  if (int rc = check_ws(who, dev_ws, ws_bytes, host_right_ws(kind, M, N, K, mode))) return rc;
  HostStreams* hs = nullptr;
  if (int rc = host_streams(&hs)) return rc;
  cudaStream_t s0 = hs->sl;  // the structured operand's stream

  // ---- X: copy in once, expand on its own stream (the A chunks' copies
  // do not wait for it; their products do)
  uint8_t* cur = static_cast<uint8_t*>(dev_ws);
  const size_t xlen = kind == HostRight::Toeplitz ? static_cast<size_t>(K) + N - 1 : static_cast<size_t>(K) * (K + 1) / 2;
  float* xraw = reinterpret_cast<float*>(cur);
  cur += right_raw_bytes(kind, N, K);
  SMM_CUDA_TRY(cudaMemcpyAsync(xraw, X, xlen * 4, cudaMemcpyHostToDevice, s0), "copy structured operand");
  Staged ex;  // the dense K x N copy (the packed expansions with K = N have the same size)
  uint8_t* xcur = cur;
  cur += toeplitz_expanded_bytes(K, N, mode);
  if (kind == HostRight::Toeplitz) {
    if (int rc = expand_toeplitz(xraw, K, N, mode, xcur, &ex, s0)) return rc;
  } else {
    if (int rc = expand_operand(xraw, kind == HostRight::Upper ? SMM_STRUCT_UPPER : SMM_STRUCT_SYMM, N, 0, N, mode,
                                xcur, &ex, s0))
      return rc;
  }
  Operand xop = dense_op(ex.ptr, nullptr, ex.ld, ex.bf16);
  if (kind == HostRight::Upper) xop.tri = 1;  // K range clipped per column tile
  SMM_CUDA_TRY(cudaEventRecord(hs->left_ready, s0), "event record");

  // ---- A in row chunks, alternating streams
  const int h = host_row_chunk(M);
  uint8_t* region[2] = {cur, cur + right_chunk_bytes(M, N, K, mode)};
  int c = 0;
  for (int r0 = 0; r0 < M; r0 += h, ++c) {
    const int k = c & 1;
    const int rows = std::min(h, M - r0);
    cudaStream_t st = hs->st[k];
    uint8_t* r = region[k];
    float* araw = reinterpret_cast<float*>(r);
    r += round256(static_cast<size_t>(h) * K * 4);
    uint8_t* stage_cur = r;
    r += staged_bytes_bound(h, K, mode);
    float* cch = reinterpret_cast<float*>(r);
    SMM_CUDA_TRY(cudaMemcpyAsync(araw, A + static_cast<size_t>(r0) * K, static_cast<size_t>(rows) * K * 4,
                                 cudaMemcpyHostToDevice, st),
                 "copy A chunk");
    Staged as;
    if (int rc = stage_operand(araw, rows, K, mode, stage_cur, &as, st)) return rc;
    if (c < 2) SMM_CUDA_TRY(cudaStreamWaitEvent(st, hs->left_ready, 0), "wait for the structured operand");
    if (c >= 2) SMM_CUDA_TRY(cudaStreamWaitEvent(st, hs->out_done[k], 0), "wait for the C buffer");
    if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(as.ptr, as.lo, as.ld, as.bf16), xop, cch,
                                 N, rows, N, K, st))
      return rc;
    // rows of C are contiguous: one copy of rows * N floats
    const size_t bytes = static_cast<size_t>(rows) * N * 4;
    if (int rc = chunk_copy_out(hs, k, C + static_cast<size_t>(r0) * N, bytes, cch, bytes, bytes, 1)) return rc;
  }
  if (int rc = drain_host_streams(hs)) return rc;
  return smm_device_status(s0);
}

}  // namespace
}  // namespace smm

using namespace smm;

extern "C" size_t smm_gen_x_upper_host_workspace_size(int M, int N, int mode) {
  return host_right_ws(HostRight::Upper, M, N, N, mode);
}
extern "C" int smm_gen_x_upper_host(const float* A, const float* U_packed, float* C, int M, int N, int mode,
                                    void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_gen_x_upper_host");
  return host_right_product("smm_gen_x_upper_host", HostRight::Upper, M, N, N, mode, A, U_packed, C, dev_ws,
                            ws_bytes);
}
extern "C" size_t smm_gen_x_symm_host_workspace_size(int M, int N, int mode) {
  return host_right_ws(HostRight::Symm, M, N, N, mode);
}
extern "C" int smm_gen_x_symm_host(const float* A, const float* S_packed, float* C, int M, int N, int mode,
                                   void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_gen_x_symm_host");
  return host_right_product("smm_gen_x_symm_host", HostRight::Symm, M, N, N, mode, A, S_packed, C, dev_ws, ws_bytes);
}
extern "C" size_t smm_gen_x_toeplitz_host_workspace_size(int M, int N, int K, int mode) {
  return host_right_ws(HostRight::Toeplitz, M, N, K, mode);
}
extern "C" int smm_gen_x_toeplitz_host(const float* A, const float* g, float* C, int M, int N, int K, int mode,
                                       void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_gen_x_toeplitz_host");
  return host_right_product("smm_gen_x_toeplitz_host", HostRight::Toeplitz, M, N, K, mode, A, g, C, dev_ws,
                            ws_bytes);
}

extern "C" size_t smm_gemm_host_workspace_size(int M, int N, int K, int mode) {
  return host_ws_bytes({HostLeft::Gemm, M, N, K, mode});
}
extern "C" int smm_gemm_host(const float* A, const float* B, float* C, int M, int N, int K, int mode, void* dev_ws,
                             size_t ws_bytes) {
  SMM_RANGE("smm_gemm_host");
  return host_product("smm_gemm_host", {HostLeft::Gemm, M, N, K, mode}, A, nullptr, B, C, dev_ws, ws_bytes);
}

extern "C" size_t smm_upper_left_host_workspace_size(int N, int ncols, int mode) {
  return host_ws_bytes({HostLeft::Upper, N, ncols, N, mode});
}
extern "C" int smm_upper_left_host(const float* U_packed, const float* B, float* C, int N, int ncols, int mode,
                                   void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_upper_left_host");
  return host_product("smm_upper_left_host", {HostLeft::Upper, N, ncols, N, mode}, U_packed, nullptr, B, C, dev_ws,
                      ws_bytes);
}

extern "C" size_t smm_symm_left_host_workspace_size(int N, int ncols, int mode) {
  return host_ws_bytes({HostLeft::Symm, N, ncols, N, mode});
}
extern "C" int smm_symm_left_host(const float* S_packed, const float* B, float* C, int N, int ncols, int mode,
                                  void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_symm_left_host");
  return host_product("smm_symm_left_host", {HostLeft::Symm, N, ncols, N, mode}, S_packed, nullptr, B, C, dev_ws,
                      ws_bytes);
}

extern "C" size_t smm_toeplitz_left_host_workspace_size(int N, int ncols, int mode) {
  return host_ws_bytes({HostLeft::Toeplitz, N, ncols, N, mode});
}
extern "C" int smm_toeplitz_left_host(const float* g, const float* B, float* C, int N, int ncols, int mode,
                                      void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_toeplitz_left_host");
  return host_product("smm_toeplitz_left_host", {HostLeft::Toeplitz, N, ncols, N, mode}, g, nullptr, B, C, dev_ws,
                      ws_bytes);
}

extern "C" size_t smm_symm_sandwich_host_workspace_size(int N, int mode) {
  return host_ws_bytes({HostLeft::Sandwich, N, N, N, mode});
}
extern "C" int smm_symm_sandwich_host(const float* A, const float* S_packed, const float* B, float* C, int N,
                                      int mode, void* dev_ws, size_t ws_bytes) {
  SMM_RANGE("smm_symm_sandwich_host");
  return host_product("smm_symm_sandwich_host", {HostLeft::Sandwich, N, N, N, mode}, A, S_packed, B, C, dev_ws,
                      ws_bytes);
}
