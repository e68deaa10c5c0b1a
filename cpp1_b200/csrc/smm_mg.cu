// Multi-GPU products: one process per GPU, NCCL over NVLink / NVSwitch.
//
// A product C = X B (X the dense A, packed U, Toeplitz generator, or A S for
// the sandwich) is partitioned by output row slabs: rank g computes rows
// [r0, r1) of C.  The shared right operand B lives on the root rank; it is
// broadcast in K-chunks (row chunks of B, contiguous in memory) on the
// communicator's high-priority stream, and the slab product is accumulated
// chunk by chunk on the caller's stream as the chunks arrive:
//   C_slab  = X[r0:r1, K_0] B[K_0, :]
//   C_slab += X[r0:r1, K_j] B[K_j, :]   (j = 1 .. c-1, each after chunk j landed)
// so the broadcast of chunk j+1 overlaps the tensor-core work on chunk j.
// Each chunk is one contraction launch with a K offset (the tensor maps start
// at the chunk; triangular and Toeplitz operands use global columns) and an
// epilogue that adds into C.  For the upper-triangular operand the chunks
// travel last-first: the slabs of the last rows need only the last rows of
// B, and they start at once.
//
// No kernel reads another GPU's memory and nothing is multicast: remote data
// reaches local HBM through NCCL before any kernel touches it.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the copy the
// process already loaded, e.g. PyTorch's), so libsmm has no link-time NCCL
// dependency and single-GPU users never load it.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "smm_contract.h"
#include "smm_host.h"

namespace smm {
namespace {

// ---------------------------------------------------------------- NCCL, resolved at run time
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = "";
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process (e.g. PyTorch's)
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      snprintf(api.why, sizeof(api.why), "libnccl.so.2 not loadable: %s", dlerror());
      return;
    }
    auto sym = [&](const char* name) { return dlsym(h, name); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(sym("ncclBroadcast"));
    api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.broadcast &&
             api.comm_get_async_error && api.error_string;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks an entry point libsmm needs");
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  const NcclApi& n = nccl();
  return set_error(SMM_ERR_NCCL, "%s: %s (%d)", what, n.error_string ? n.error_string(r) : "NCCL error", int(r));
}

#define SMM_NCCL_TRY(expr, what)                          \
  do {                                                    \
    ncclResult_t _r = (expr);                             \
    if (_r != ncclSuccess) return nccl_fail(_r, what);    \
  } while (0)

constexpr int kMaxChunks = 16;

}  // namespace
}  // namespace smm

// One rank's communicator: the NCCL communicator, the device it was created
// on, a high-priority stream for the collectives and the events that order
// them against the caller's stream.
struct smm_mg_comm {
  ncclComm_t nc = nullptr;
  int rank = 0;
  int world = 1;
  int device = 0;
  cudaStream_t cs = nullptr;
  cudaEvent_t ev_start = nullptr;
  cudaEvent_t ev_chunk[smm::kMaxChunks] = {};
};

namespace smm {
namespace {

// ---------------------------------------------------------------- partition
long long range_cost(long long n, long long a, long long b) {  // sum_{i=a}^{b-1} (n - i)
  return (b - a) * n - (b * (b - 1) - a * (a - 1)) / 2;
}

// Slab boundaries b[0] = 0 <= ... <= b[world] = n on 128-row tiles,
// minimising the largest slab's work: rows cost 1 (dense operands) or n - i
// (upper-triangular).  Binary search on the largest slab's work, then a
// greedy cut.  Slabs may be empty when n has fewer tiles than ranks.
void row_slabs(int n, int world, bool triangular, int* b) {
  constexpr int kTile = 128;
  if (n <= 0) {
    for (int g = 0; g <= world; ++g) b[g] = 0;
    return;
  }
  const int tiles = (n + kTile - 1) / kTile;
  std::vector<long long> w(tiles);
  for (int t = 0; t < tiles; ++t) {
    const int a = t * kTile, e = std::min(n, (t + 1) * kTile);
    w[t] = triangular ? range_cost(n, a, e) : (e - a);
  }
  auto groups = [&](long long cap) {
    int count = 1;
    long long acc = 0;
    for (long long x : w) {
      if (acc + x > cap) {
        ++count;
        acc = x;
      } else {
        acc += x;
      }
    }
    return count;
  };
  long long lo = *std::max_element(w.begin(), w.end()), hi = 0;
  for (long long x : w) hi += x;
  while (lo < hi) {
    const long long mid = (lo + hi) / 2;
    if (groups(mid) <= world)
      hi = mid;
    else
      lo = mid + 1;
  }
  std::vector<int> cuts{0};
  long long acc = 0;
  for (int t = 0; t < tiles; ++t) {
    if (acc + w[t] > lo) {
      cuts.push_back(t * kTile);
      acc = w[t];
    } else {
      acc += w[t];
    }
  }
  cuts.push_back(n);
  while (static_cast<int>(cuts.size()) < world + 1) cuts.insert(cuts.end() - 1, n);
  for (int g = 0; g <= world; ++g) b[g] = cuts[g];
}

// K-chunk boundaries of a broadcast of k rows: about k / 1024 chunks (2 to 8;
// SMM_MG_CHUNKS overrides, 1 .. 15), multiples of 256 rows.
int chunk_bounds(int k, int world, int* kb) {
  int c = 1;
  if (world > 1) {
    c = std::min(8, std::max(2, k / 1024));
    if (const char* e = std::getenv("SMM_MG_CHUNKS")) {
      const int v = std::atoi(e);
      if (v >= 1 && v < kMaxChunks) c = v;  // the last event slot is the sandwich's S
    }
  }
  int per = (k + c - 1) / c;
  per = (per + 255) / 256 * 256;
  int n = 0;
  kb[0] = 0;
  for (int a = 0; a < k; a += per) kb[++n] = std::min(k, a + per);
  if (n == 0) kb[++n] = k;  // k == 0
  return n;
}

int check_comm(const smm_mg_comm* c, const char* who) {
  if (!c) return set_error(SMM_ERR_INVALID, "%s: null communicator", who);
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != c->device)
    return set_error(SMM_ERR_INVALID, "%s: current device %d is not the communicator's device %d", who, dev,
                     c->device);
  return SMM_OK;
}

// The chunked broadcast: the comm stream waits for the caller's stream (B and
// the previous call's readers are done), then broadcasts chunk j (in `order`)
// and records ev_chunk[j] after it.
int broadcast_chunks(smm_mg_comm* c, float* B, int ld, const int* kb, int nch, const int* order, int root,
                     cudaStream_t st) {
  if (c->world == 1) return SMM_OK;
  SMM_CUDA_TRY(cudaEventRecord(c->ev_start, st), "record call start");
  SMM_CUDA_TRY(cudaStreamWaitEvent(c->cs, c->ev_start, 0), "order broadcast after the caller's stream");
  const NcclApi& n = nccl();
  for (int q = 0; q < nch; ++q) {
    const int j = order[q];
    float* p = B + static_cast<size_t>(kb[j]) * ld;
    const size_t count = static_cast<size_t>(kb[j + 1] - kb[j]) * ld;
    SMM_NCCL_TRY(n.broadcast(p, p, count, ncclFloat, root, c->nc, c->cs), "ncclBroadcast (K-chunk of B)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_chunk[j], c->cs), "record chunk arrival");
  }
  return SMM_OK;
}

int wait_chunk(smm_mg_comm* c, int j, cudaStream_t st) {
  if (c->world == 1) return SMM_OK;
  SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_chunk[j], 0), "wait for chunk arrival");
  return SMM_OK;
}

// The B chunk as a contraction operand: fp32 in place (rows 16-byte aligned),
// or its bf16 copy converted into rows [kb[j], kb[j+1]) of the bf16 plane
// `bf` (bf16 mode) once it has arrived.
int chunk_operand(const float* B, int ld, __nv_bfloat16* bf, int ldb, int k0, int k1, int mode, cudaStream_t st,
                  Operand* out) {
  const float* src = B + static_cast<size_t>(k0) * ld;
  if (mode == SMM_MODE_BF16) {
    uint8_t* cur = reinterpret_cast<uint8_t*>(bf + static_cast<size_t>(k0) * ldb);
    Staged s;
    if (int rc = stage_operand(src, k1 - k0, ld, mode, cur, &s, st)) return rc;
    *out = dense_op(nullptr, nullptr, s.ld, s.bf16);
  } else {
    *out = dense_op(src, nullptr, ld);
  }
  return SMM_OK;
}

bool aligned_rows(const float* p, int ld) { return aligned16(p) && ld % 4 == 0; }

}  // namespace
}  // namespace smm

using namespace smm;

// ---------------------------------------------------------------- C ABI
extern "C" int smm_mg_unique_id(void* id_out) {
  SMM_RANGE("smm_mg_unique_id");
  if (!id_out) return set_error(SMM_ERR_INVALID, "smm_mg_unique_id: null output");
  const NcclApi& n = nccl();
  if (!n.ok) return set_error(SMM_ERR_NCCL, "%s", n.why);
  ncclUniqueId id;
  SMM_NCCL_TRY(n.get_unique_id(&id), "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == SMM_MG_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, &id, sizeof(id));
  return SMM_OK;
}

extern "C" int smm_mg_comm_init(smm_mg_comm** out, int rank, int world, const void* id) {
  SMM_RANGE("smm_mg_comm_init");
  if (!out) return set_error(SMM_ERR_INVALID, "smm_mg_comm_init: null output");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return set_error(SMM_ERR_INVALID, "smm_mg_comm_init: rank %d of %d", rank, world);
  if (world > 1 && !id) return set_error(SMM_ERR_INVALID, "smm_mg_comm_init: null unique id");
  auto* c = new smm_mg_comm();
  c->rank = rank;
  c->world = world;
  auto fail = [&](int rc) {
    if (c->cs) cudaStreamDestroy(c->cs);
    if (c->ev_start) cudaEventDestroy(c->ev_start);
    for (auto& e : c->ev_chunk)
      if (e) cudaEventDestroy(e);
    delete c;
    return rc;
  };
  if (cudaGetDevice(&c->device) != cudaSuccess) return fail(set_error(SMM_ERR_CUDA, "cudaGetDevice failed"));
  int lo = 0, hi = 0;
  if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
      cudaStreamCreateWithPriority(&c->cs, cudaStreamNonBlocking, hi) != cudaSuccess)
    return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: collective stream"));
  if (cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming) != cudaSuccess)
    return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  for (auto& e : c->ev_chunk)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  if (world > 1) {
    const NcclApi& n = nccl();
    if (!n.ok) return fail(set_error(SMM_ERR_NCCL, "%s", n.why));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = n.comm_init_rank(&c->nc, world, uid, rank);
    if (r != ncclSuccess) return fail(nccl_fail(r, "ncclCommInitRank"));
  }
  *out = c;
  return SMM_OK;
}

extern "C" int smm_mg_comm_destroy(smm_mg_comm* c) {
  SMM_RANGE("smm_mg_comm_destroy");
  if (!c) return SMM_OK;
  int rc = SMM_OK;
  if (c->cs) cudaStreamSynchronize(c->cs);
  if (c->nc) {
    ncclResult_t r = nccl().comm_destroy(c->nc);
    if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommDestroy");
  }
  if (c->cs) cudaStreamDestroy(c->cs);
  if (c->ev_start) cudaEventDestroy(c->ev_start);
  for (auto& e : c->ev_chunk)
    if (e) cudaEventDestroy(e);
  delete c;
  return rc;
}

extern "C" int smm_mg_comm_abort(smm_mg_comm* c) {
  SMM_RANGE("smm_mg_comm_abort");
  if (!c) return SMM_OK;
  int rc = SMM_OK;
  if (c->nc) {
    ncclResult_t r = nccl().comm_abort(c->nc);
    if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommAbort");
  }
  if (c->cs) cudaStreamDestroy(c->cs);
  if (c->ev_start) cudaEventDestroy(c->ev_start);
  for (auto& e : c->ev_chunk)
    if (e) cudaEventDestroy(e);
  delete c;
  return rc;
}

extern "C" int smm_mg_comm_status(smm_mg_comm* c) {
  if (!c) return set_error(SMM_ERR_INVALID, "smm_mg_comm_status: null communicator");
  if (!c->nc) return SMM_OK;
  ncclResult_t a = ncclSuccess;
  SMM_NCCL_TRY(nccl().comm_get_async_error(c->nc, &a), "ncclCommGetAsyncError");
  if (a != ncclSuccess && a != ncclInProgress) return nccl_fail(a, "asynchronous NCCL error");
  return SMM_OK;
}

extern "C" int smm_mg_row_slabs(int N, int world, int triangular, int* bounds) {
  if (N < 0 || world < 1 || !bounds) return set_error(SMM_ERR_INVALID, "smm_mg_row_slabs: bad arguments");
  row_slabs(N, world, triangular != 0, bounds);
  return SMM_OK;
}

extern "C" int smm_mg_chunks(int K, int world, int* bounds) {
  if (K < 0 || world < 1 || !bounds) return set_error(SMM_ERR_INVALID, "smm_mg_chunks: bad arguments");
  return chunk_bounds(K, world, bounds);
}

// ---------------------------------------------------------------- products
extern "C" size_t smm_mg_gemm_workspace_size(int nrows, int N, int K, int mode) {
  if (nrows <= 0 || N <= 0 || K <= 0) return 0;
  // the A slab staged (bf16 copy, or a padded fp32 copy) + B's bf16 plane
  return staged_bytes_bound(nrows, K, mode) + (mode == SMM_MODE_BF16 ? bf16_plane_bytes(K, N) : 0);
}

extern "C" int smm_mg_gemm(smm_mg_comm* c, const float* A_slab, float* B, float* C_slab, int nrows, int N, int K,
                           int mode, int root, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_gemm");
  if (int rc = check_comm(c, "smm_mg_gemm")) return rc;
  if (nrows < 0 || N < 0 || K < 0 || root < 0 || root >= c->world)
    return set_error(SMM_ERR_INVALID, "smm_mg_gemm: bad shape or root");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: unknown mode %d", mode);
  if (N == 0 || K == 0) return SMM_OK;
  if (!B || (nrows > 0 && (!A_slab || !C_slab))) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: null pointer");
  if (!aligned_rows(B, N)) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: B needs 16-byte aligned rows");
  cudaStream_t st = as_stream(stream);
  int kb[kMaxChunks + 1], order[kMaxChunks];
  const int nch = chunk_bounds(K, c->world, kb);
  for (int j = 0; j < nch; ++j) order[j] = j;
  if (int rc = broadcast_chunks(c, B, N, kb, nch, order, root, st)) return rc;
  if (nrows == 0) return SMM_OK;
  const size_t need = staged_bytes(A_slab, nrows, K, mode) + (mode == SMM_MODE_BF16 ? bf16_plane_bytes(K, N) : 0);
  if (int rc = check_ws("smm_mg_gemm", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged a;
  if (int rc = stage_operand(A_slab, nrows, K, mode, cur, &a, st)) return rc;
  __nv_bfloat16* bbf = mode == SMM_MODE_BF16 ? reinterpret_cast<__nv_bfloat16*>(cur) : nullptr;
  const int ldb = round8(N);
  for (int q = 0; q < nch; ++q) {
    const int j = order[q];
    if (int rc = wait_chunk(c, j, st)) return rc;
    Operand bo;
    if (int rc = chunk_operand(B, N, bbf, ldb, kb[j], kb[j + 1], mode, st, &bo)) return rc;
    const size_t off = static_cast<size_t>(kb[j]);
    Operand ao = dense_op(a.ptr ? a.ptr + off : nullptr, nullptr, a.ld, a.bf16 ? a.bf16 + off : nullptr);
    ao.k_off = kb[j];
    if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, ao, bo, C_slab, N, nrows, N, kb[j + 1] - kb[j], st,
                                 nullptr, nullptr, 0, q > 0))
      return rc;
  }
  return SMM_OK;
}

extern "C" size_t smm_mg_upper_left_workspace_size(int N, int ncols, int row0, int nrows, int mode) {
  if (N <= 0 || ncols <= 0 || nrows <= 0) return 0;
  (void)row0;
  return expanded_bytes(nrows, N, mode) + (mode == SMM_MODE_BF16 ? bf16_plane_bytes(N, ncols) : 0);
}

extern "C" int smm_mg_upper_left(smm_mg_comm* c, const float* U_packed, float* B, float* C_slab, int N, int ncols,
                                 int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_upper_left");
  if (int rc = check_comm(c, "smm_mg_upper_left")) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N || root < 0 || root >= c->world)
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: bad shape, slab or root");
  if (int rc = check_packed("smm_mg_upper_left", N)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: unknown mode %d", mode);
  if (N == 0 || ncols == 0) return SMM_OK;
  if (!B || (nrows > 0 && (!U_packed || !C_slab)))
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: null pointer");
  if (!aligned_rows(B, ncols)) return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: B needs 16-byte aligned rows");
  cudaStream_t st = as_stream(stream);
  int kb[kMaxChunks + 1], order[kMaxChunks];
  const int nch = chunk_bounds(N, c->world, kb);
  for (int q = 0; q < nch; ++q) order[q] = nch - 1 - q;  // last rows of B first
  if (int rc = broadcast_chunks(c, B, ncols, kb, nch, order, root, st)) return rc;
  if (nrows == 0) return SMM_OK;
  const size_t need = expanded_bytes(nrows, N, mode) + (mode == SMM_MODE_BF16 ? bf16_plane_bytes(N, ncols) : 0);
  if (int rc = check_ws("smm_mg_upper_left", ws, ws_bytes, need)) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  Staged u;  // rows [row0, row0 + nrows) of U, dense (zeros left of the diagonal)
  if (int rc = expand_operand(U_packed, SMM_STRUCT_UPPER, N, row0, nrows, mode, cur, &u, st)) return rc;
  __nv_bfloat16* bbf = mode == SMM_MODE_BF16 ? reinterpret_cast<__nv_bfloat16*>(cur) : nullptr;
  const int ldb = round8(ncols);
  bool first = true;
  for (int q = 0; q < nch; ++q) {
    const int j = order[q];
    if (int rc = wait_chunk(c, j, st)) return rc;
    if (kb[j + 1] <= row0) continue;  // this slab's rows are zero there (the chunk is still received)
    Operand bo;
    if (int rc = chunk_operand(B, ncols, bbf, ldb, kb[j], kb[j + 1], mode, st, &bo)) return rc;
    const size_t off = static_cast<size_t>(kb[j]);
    Operand ao = dense_op(u.ptr ? u.ptr + off : nullptr, nullptr, u.ld, u.bf16 ? u.bf16 + off : nullptr);
    ao.dim = N;
    ao.row0 = row0;
    ao.k_off = kb[j];
    if (int rc = run_contraction(AKind::UpperDense, BKind::Dense, mode, ao, bo, C_slab, ncols, nrows, ncols,
                                 kb[j + 1] - kb[j], st, nullptr, nullptr, 0, !first))
      return rc;
    first = false;
  }
  return SMM_OK;
}

extern "C" size_t smm_mg_toeplitz_left_workspace_size(int N, int ncols, int mode) {
  if (N <= 0 || ncols <= 0) return 0;
  return mode == SMM_MODE_BF16 ? bf16_plane_bytes(N, ncols) : 0;
}

extern "C" int smm_mg_toeplitz_left(smm_mg_comm* c, const float* g, float* B, float* C_slab, int N, int ncols,
                                    int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes,
                                    void* stream) {
  SMM_RANGE("smm_mg_toeplitz_left");
  if (int rc = check_comm(c, "smm_mg_toeplitz_left")) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N || root < 0 || root >= c->world)
    return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: bad shape, slab or root");
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: unknown mode %d", mode);
  if (N == 0 || ncols == 0) return SMM_OK;
  if (!B || (nrows > 0 && (!g || !C_slab))) return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: null pointer");
  if (!aligned_rows(B, ncols))
    return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: B needs 16-byte aligned rows");
  cudaStream_t st = as_stream(stream);
  int kb[kMaxChunks + 1], order[kMaxChunks];
  const int nch = chunk_bounds(N, c->world, kb);
  for (int j = 0; j < nch; ++j) order[j] = j;
  if (int rc = broadcast_chunks(c, B, ncols, kb, nch, order, root, st)) return rc;
  if (nrows == 0) return SMM_OK;
  const size_t need = mode == SMM_MODE_BF16 ? bf16_plane_bytes(N, ncols) : 0;
  if (int rc = check_ws("smm_mg_toeplitz_left", ws, ws_bytes, need)) return rc;
  __nv_bfloat16* bbf = mode == SMM_MODE_BF16 ? static_cast<__nv_bfloat16*>(ws) : nullptr;
  const int ldb = round8(ncols);
  for (int q = 0; q < nch; ++q) {
    const int j = order[q];
    if (int rc = wait_chunk(c, j, st)) return rc;
    Operand bo;
    if (int rc = chunk_operand(B, ncols, bbf, ldb, kb[j], kb[j + 1], mode, st, &bo)) return rc;
    Operand ao = structured_op(g, N, row0);
    ao.k_off = kb[j];
    if (int rc = run_contraction(AKind::Toeplitz, BKind::Dense, mode, ao, bo, C_slab, ncols, nrows, ncols,
                                 kb[j + 1] - kb[j], st, nullptr, nullptr, 0, q > 0))
      return rc;
  }
  return SMM_OK;
}

namespace {
// Sandwich workspace: Y = A_slab S (fp32, 16-byte rows; plus its bf16 copy in
// bf16 mode), the dense expansion of S, the staged A slab, B's bf16 plane.
size_t mg_sandwich_ws(int N, int nrows, int mode) {
  const bool bf = mode == SMM_MODE_BF16;
  return plane_bytes(nrows, N) + (bf ? bf16_plane_bytes(nrows, N) : 0) + expanded_bytes(N, N, mode) +
         staged_bytes_bound(nrows, N, mode) + (bf ? bf16_plane_bytes(N, N) : 0);
}
}  // namespace

extern "C" size_t smm_mg_symm_sandwich_workspace_size(int N, int nrows, int mode) {
  if (N <= 0 || nrows <= 0) return 0;
  return mg_sandwich_ws(N, nrows, mode);
}

extern "C" int smm_mg_symm_sandwich(smm_mg_comm* c, const float* A_slab, float* S_packed, float* B, float* C_slab,
                                    int N, int nrows, int mode, int root, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_symm_sandwich");
  if (int rc = check_comm(c, "smm_mg_symm_sandwich")) return rc;
  if (N < 0 || nrows < 0 || nrows > N || root < 0 || root >= c->world)
    return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: bad shape or root");
  if (int rc = check_packed("smm_mg_symm_sandwich", N)) return rc;
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: unknown mode %d", mode);
  if (N == 0) return SMM_OK;
  if (!S_packed || !B || (nrows > 0 && (!A_slab || !C_slab)))
    return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: null pointer");
  if (!aligned_rows(B, N)) return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: B needs 16-byte aligned rows");
  cudaStream_t st = as_stream(stream);
  const bool bf = mode == SMM_MODE_BF16;
  // S travels whole first (packed, N(N+1)/2 floats), then B in K-chunks.
  int kb[kMaxChunks + 2], order[kMaxChunks];
  const int nch = chunk_bounds(N, c->world, kb);
  for (int j = 0; j < nch; ++j) order[j] = j;
  if (c->world > 1) {
    SMM_CUDA_TRY(cudaEventRecord(c->ev_start, st), "record call start");
    SMM_CUDA_TRY(cudaStreamWaitEvent(c->cs, c->ev_start, 0), "order broadcast after the caller's stream");
    const size_t ns = static_cast<size_t>(N) * (N + 1) / 2;
    SMM_NCCL_TRY(nccl().broadcast(S_packed, S_packed, ns, ncclFloat, root, c->nc, c->cs), "ncclBroadcast (S)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_chunk[kMaxChunks - 1], c->cs), "record S arrival");
    const NcclApi& n = nccl();
    for (int q = 0; q < nch; ++q) {
      const int j = order[q];
      float* p = B + static_cast<size_t>(kb[j]) * N;
      SMM_NCCL_TRY(n.broadcast(p, p, static_cast<size_t>(kb[j + 1] - kb[j]) * N, ncclFloat, root, c->nc, c->cs),
                   "ncclBroadcast (K-chunk of B)");
      SMM_CUDA_TRY(cudaEventRecord(c->ev_chunk[j], c->cs), "record chunk arrival");
    }
  }
  if (nrows == 0) return SMM_OK;
  if (int rc = check_ws("smm_mg_symm_sandwich", ws, ws_bytes, mg_sandwich_ws(N, nrows, mode))) return rc;
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* Y = reinterpret_cast<float*>(cur);
  const int ldy = round4(N), ldy_bf = round8(N);
  cur += plane_bytes(nrows, N);
  __nv_bfloat16* Y_bf = nullptr;
  if (bf) {
    Y_bf = reinterpret_cast<__nv_bfloat16*>(cur);
    cur += bf16_plane_bytes(nrows, N);
    if (ldy_bf != N) SMM_CUDA_TRY(cudaMemsetAsync(Y_bf, 0, bf16_plane_bytes(nrows, N), st), "zero bf16 rows");
  }
  Staged a;
  if (int rc = stage_operand(A_slab, nrows, N, mode, cur, &a, st)) return rc;
  if (c->world > 1) SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_chunk[kMaxChunks - 1], 0), "wait for S");
  Staged s;  // S mirrored into a dense copy: the right operand of Y = A_slab S
  if (int rc = expand_operand(S_packed, SMM_STRUCT_SYMM, N, 0, N, mode, cur, &s, st)) return rc;
  if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, nullptr, a.ld, a.bf16),
                               dense_op(s.ptr, nullptr, s.ld, s.bf16), Y, ldy, nrows, N, N, st, nullptr, Y_bf,
                               ldy_bf))
    return rc;
  __nv_bfloat16* bbf = bf ? reinterpret_cast<__nv_bfloat16*>(cur) : nullptr;
  const int ldb = round8(N);
  for (int q = 0; q < nch; ++q) {
    const int j = order[q];
    if (int rc = wait_chunk(c, j, st)) return rc;
    Operand bo;
    if (int rc = chunk_operand(B, N, bbf, ldb, kb[j], kb[j + 1], mode, st, &bo)) return rc;
    const size_t off = static_cast<size_t>(kb[j]);
    Operand yo = dense_op(bf ? nullptr : Y + off, nullptr, bf ? ldy_bf : ldy, bf ? Y_bf + off : nullptr);
    yo.k_off = kb[j];
    if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, yo, bo, C_slab, N, nrows, N, kb[j + 1] - kb[j], st,
                                 nullptr, nullptr, 0, q > 0))
      return rc;
  }
  return SMM_OK;
}
