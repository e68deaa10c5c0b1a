// Multi-GPU products: one process per GPU, NCCL over NVLink / NVSwitch.
//
// A product C = X B (X the dense A, packed U, Toeplitz generator, or A S for
// the sandwich) is partitioned by output row slabs: rank g computes rows
// [r0, r1) of C.  The shared right operand B lives on the root rank and is
// broadcast inside each call in COLUMN blocks: the root copies column block
// j of B into a contiguous K x W_j buffer and broadcasts it on the
// communicator's high-priority stream; every rank computes
//   C_slab[:, block j] = X[r0:r1, :] B[:, block j]
// from that buffer as soon as it has landed, on one of several internal
// compute streams, so block j's tensor-core work overlaps the transfer of the
// blocks after it, and blocks that arrive while earlier ones still compute
// run side by side.  Every output element is written once by one full-K
// contraction (no partial sums: results identical to the single-GPU entry
// points).
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
constexpr int kWork = 4;  // internal compute streams

}  // namespace
}  // namespace smm

// One rank's communicator: the NCCL communicator, the device it was created
// on, a high-priority stream for the collectives, the compute streams the
// column blocks run on, and the events that order them against the caller's
// stream.
struct smm_mg_comm {
  ncclComm_t nc = nullptr;
  int rank = 0;
  int world = 1;
  int device = 0;
  cudaStream_t cs = nullptr;
  cudaStream_t work[smm::kWork] = {};
  cudaEvent_t ev_start = nullptr;  // caller's stream: inputs ready, previous call's readers done
  cudaEvent_t ev_prep = nullptr;   // caller's stream: the left operand prepared
  cudaEvent_t ev_s = nullptr;      // collective stream: the sandwich's S arrived
  cudaEvent_t ev_chunk[smm::kMaxChunks] = {};
  cudaEvent_t ev_done[smm::kWork] = {};
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

// Column block [c0, c0 + w) of B (K x ncols, 16-byte aligned rows; c0 and
// ncols multiples of 4) into the contiguous K x w buffer dst: 128-bit loads
// and stores, a grid-stride loop over the block's float4 quads.  An SM copy
// at HBM speed; a strided cudaMemcpy2D of the same block measured ~3x slower.
__global__ void __launch_bounds__(256) pack_cols_kernel(const float* __restrict__ B, int ncols, int c0, int K, int w,
                                                        float* __restrict__ dst) {
  const int wq = (w + 3) / 4;
  const long long total = static_cast<long long>(K) * wq;
  for (long long q = blockIdx.x * 256LL + threadIdx.x; q < total; q += static_cast<long long>(gridDim.x) * 256) {
    const int k = static_cast<int>(q / wq), j = 4 * static_cast<int>(q - static_cast<long long>(k) * wq);
    const float* s = B + static_cast<long long>(k) * ncols + c0 + j;
    float* d = dst + static_cast<long long>(k) * w + j;
    if (j + 4 <= w && (w & 3) == 0) {
      *reinterpret_cast<float4*>(d) = __ldcs(reinterpret_cast<const float4*>(s));
    } else {
      for (int e = 0; e < 4 && j + e < w; ++e) d[e] = s[e];
    }
  }
}

// Column-block boundaries of a broadcast of B (ncols columns): 1 block at
// world 1, else 4 (SMM_MG_CHUNKS overrides, 1 .. 16), widths multiples of 256
// (the widest output tile).
int chunk_bounds(int ncols, int world, int* cb) {
  int c = 1;
  if (world > 1) {
    c = 4;
    if (const char* e = std::getenv("SMM_MG_CHUNKS")) {
      const int v = std::atoi(e);
      if (v >= 1 && v <= kMaxChunks) c = v;
    }
  }
  int per = (ncols + c - 1) / c;
  per = std::max(256, (per + 255) / 256 * 256);
  int n = 0;
  cb[0] = 0;
  for (int a = 0; a < ncols; a += per) cb[++n] = std::min(ncols, a + per);
  if (n == 0) cb[++n] = ncols;  // ncols == 0
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

// Workspace of the B side: the packed column blocks (world > 1) and, in bf16
// mode, their bf16 copies (one plane per block; at world 1 one plane of B).
size_t b_side_bytes(int world, int K, int ncols, int mode) {
  int cb[kMaxChunks + 1];
  const int nch = chunk_bounds(ncols, world, cb);
  size_t b = world > 1 ? round256(static_cast<size_t>(K) * ncols * 4) : 0;
  if (mode == SMM_MODE_BF16)
    for (int j = 0; j < nch; ++j) b += bf16_plane_bytes(K, cb[j + 1] - cb[j]);
  return b;
}

// The B side of one call.  world > 1: the collective stream waits for the
// caller's stream, then per block j the root packs B[:, block j] into its
// K x W_j buffer (contiguous, at offset K * cb[j] of `pack`) and every rank
// receives it there; ev_chunk[j] marks its arrival.  (The sandwich's
// S_packed, s_count floats, is broadcast first, marked by ev_s.)
int broadcast_blocks(smm_mg_comm* c, const float* B, int K, int ncols, float* pack, const int* cb, int nch, int root,
                     cudaStream_t st, float* S_packed = nullptr, size_t s_count = 0) {
  if (c->world == 1) return SMM_OK;
  SMM_CUDA_TRY(cudaEventRecord(c->ev_start, st), "record call start");
  SMM_CUDA_TRY(cudaStreamWaitEvent(c->cs, c->ev_start, 0), "order broadcast after the caller's stream");
  const NcclApi& n = nccl();
  if (S_packed) {
    SMM_NCCL_TRY(n.broadcast(S_packed, S_packed, s_count, ncclFloat, root, c->nc, c->cs), "ncclBroadcast (S)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_s, c->cs), "record S arrival");
  }
  // The root packs every block first: the packs are enqueued before its own
  // slab's contractions, so they take the SMs at once instead of competing
  // with them between broadcasts.
  if (c->rank == root) {
    for (int j = 0; j < nch; ++j) {
      pack_cols_kernel<<<148 * 4, 256, 0, c->cs>>>(B, ncols, cb[j], K, cb[j + 1] - cb[j],
                                                   pack + static_cast<size_t>(K) * cb[j]);
      count_launch();
      SMM_CUDA_TRY(cudaGetLastError(), "pack column block of B");
    }
  }
  for (int j = 0; j < nch; ++j) {
    const int w = cb[j + 1] - cb[j];
    float* blk = pack + static_cast<size_t>(K) * cb[j];
    SMM_NCCL_TRY(n.broadcast(blk, blk, static_cast<size_t>(K) * w, ncclFloat, root, c->nc, c->cs),
                 "ncclBroadcast (column block of B)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_chunk[j], c->cs), "record block arrival");
  }
  return SMM_OK;
}

// Runs block(j, stream) for every column block: at world 1 the single block
// on the caller's stream; else block j on compute stream j % kWork once the
// left operand is prepared (ev_prep, recorded on the caller's stream) and,
// with wait_blocks, the block has landed; the caller's stream then waits for
// all of them.
template <typename F>
int run_blocks(smm_mg_comm* c, int nch, cudaStream_t st, bool wait_blocks, F&& block) {
  if (c->world == 1) return block(0, st);
  SMM_CUDA_TRY(cudaEventRecord(c->ev_prep, st), "record operand preparation");
  const int used = std::min(nch, kWork);
  for (int w = 0; w < used; ++w) SMM_CUDA_TRY(cudaStreamWaitEvent(c->work[w], c->ev_prep, 0), "fork");
  for (int j = 0; j < nch; ++j) {
    cudaStream_t w = c->work[j % kWork];
    if (wait_blocks) SMM_CUDA_TRY(cudaStreamWaitEvent(w, c->ev_chunk[j], 0), "wait for block arrival");
    if (int rc = block(j, w)) return rc;
  }
  for (int w = 0; w < used; ++w) {
    SMM_CUDA_TRY(cudaEventRecord(c->ev_done[w], c->work[w]), "record block done");
    SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_done[w], 0), "join");
  }
  return SMM_OK;
}

// Whether column block j's contraction must wait for the block's broadcast:
// the root reads its own B in place in the fp32 modes (bf16 converts the
// packed block).
bool waits_for_blocks(const smm_mg_comm* c, int root, int mode) { return c->rank != root || mode == SMM_MODE_BF16; }

// The B operand of column block j (K x W_j): fp32 in place (the caller's B at
// world 1 and on the root, the received block otherwise), or its bf16 copy
// converted on `st` into the block's bf16 plane.
int block_operand(const smm_mg_comm* c, const float* B, int K, int ncols, const float* pack, const int* cb, int j,
                  int mode, uint8_t* bf_base, cudaStream_t st, Operand* out, int root) {
  const int w = cb[j + 1] - cb[j];
  if (mode != SMM_MODE_BF16) {
    if (c->world == 1 || c->rank == root)
      *out = dense_op(B + cb[j], nullptr, ncols);
    else
      *out = dense_op(pack + static_cast<size_t>(K) * cb[j], nullptr, w);
    return SMM_OK;
  }
  const float* src = c->world == 1 ? B : pack + static_cast<size_t>(K) * cb[j];
  uint8_t* cur = bf_base;
  for (int i = 0; i < j; ++i) cur += bf16_plane_bytes(K, cb[i + 1] - cb[i]);
  Staged s;
  if (int rc = stage_operand(src, K, w, mode, cur, &s, st)) return rc;
  *out = dense_op(nullptr, nullptr, s.ld, s.bf16);
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

namespace {
void release(smm_mg_comm* c) {
  if (c->cs) cudaStreamDestroy(c->cs);
  for (auto& w : c->work)
    if (w) cudaStreamDestroy(w);
  for (cudaEvent_t e : {c->ev_start, c->ev_prep, c->ev_s})
    if (e) cudaEventDestroy(e);
  for (auto& e : c->ev_chunk)
    if (e) cudaEventDestroy(e);
  for (auto& e : c->ev_done)
    if (e) cudaEventDestroy(e);
  delete c;
}
}  // namespace

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
    release(c);
    return rc;
  };
  if (cudaGetDevice(&c->device) != cudaSuccess) return fail(set_error(SMM_ERR_CUDA, "cudaGetDevice failed"));
  int lo = 0, hi = 0;
  if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
      cudaStreamCreateWithPriority(&c->cs, cudaStreamNonBlocking, hi) != cudaSuccess)
    return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: collective stream"));
  for (auto& w : c->work)
    if (cudaStreamCreateWithFlags(&w, cudaStreamNonBlocking) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: compute stream"));
  for (cudaEvent_t* e : {&c->ev_start, &c->ev_prep, &c->ev_s})
    if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  for (auto& e : c->ev_chunk)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  for (auto& e : c->ev_done)
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
  for (auto& w : c->work)
    if (w) cudaStreamSynchronize(w);
  if (c->nc) {
    ncclResult_t r = nccl().comm_destroy(c->nc);
    if (r != ncclSuccess) rc = nccl_fail(r, "ncclCommDestroy");
  }
  release(c);
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
  release(c);
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

extern "C" int smm_mg_chunks(int ncols, int world, int* bounds) {
  if (ncols < 0 || world < 1 || !bounds) return set_error(SMM_ERR_INVALID, "smm_mg_chunks: bad arguments");
  return chunk_bounds(ncols, world, bounds);
}

namespace {
// Validation shared by the products.
int check_call(const smm_mg_comm* c, const char* who, int mode, int root, const float* B, int ncols) {
  if (int rc = check_comm(c, who)) return rc;
  if (root < 0 || root >= c->world) return set_error(SMM_ERR_INVALID, "%s: root %d of %d", who, root, c->world);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  if (c->rank == root && (!B || !aligned_rows(B, ncols)))
    return set_error(SMM_ERR_INVALID, "%s: the root's B must be non-null with 16-byte aligned rows", who);
  return SMM_OK;
}
}  // namespace

// ---------------------------------------------------------------- products
extern "C" size_t smm_mg_gemm_workspace_size(const smm_mg_comm* c, int nrows, int N, int K, int mode) {
  if (!c || nrows < 0 || N <= 0 || K <= 0) return 0;
  return b_side_bytes(c->world, K, N, mode) + (nrows ? staged_bytes_bound(nrows, K, mode) : 0);
}

extern "C" int smm_mg_gemm(smm_mg_comm* c, const float* A_slab, const float* B, float* C_slab, int nrows, int N,
                           int K, int mode, int root, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_gemm");
  if (int rc = check_call(c, "smm_mg_gemm", mode, root, B, N)) return rc;
  if (nrows < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: negative shape");
  if (N == 0 || K == 0) return SMM_OK;
  if (nrows > 0 && (!A_slab || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: null pointer");
  if (int rc = check_ws("smm_mg_gemm", ws, ws_bytes, smm_mg_gemm_workspace_size(c, nrows, N, K, mode))) return rc;
  cudaStream_t st = as_stream(stream);
  int cb[kMaxChunks + 1];
  const int nch = chunk_bounds(N, c->world, cb);
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* pack = reinterpret_cast<float*>(cur);
  uint8_t* bf = cur + (c->world > 1 ? round256(static_cast<size_t>(K) * N * 4) : 0);
  cur += b_side_bytes(c->world, K, N, mode);
  if (int rc = broadcast_blocks(c, B, K, N, pack, cb, nch, root, st)) return rc;
  Staged a{};
  if (nrows > 0)
    if (int rc = stage_operand(A_slab, nrows, K, mode, cur, &a, st)) return rc;
  return run_blocks(c, nch, st, waits_for_blocks(c, root, mode), [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    Operand bo;
    if (int rc = block_operand(c, B, K, N, pack, cb, j, mode, bf, w, &bo, root)) return rc;
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, nullptr, a.ld, a.bf16), bo,
                           C_slab + cb[j], N, nrows, cb[j + 1] - cb[j], K, w, nullptr, nullptr, 0, true);
  });
}

extern "C" size_t smm_mg_upper_left_workspace_size(const smm_mg_comm* c, int N, int ncols, int nrows, int mode) {
  if (!c || N <= 0 || ncols <= 0 || nrows < 0) return 0;
  return b_side_bytes(c->world, N, ncols, mode) + (nrows ? expanded_bytes(nrows, N, mode) : 0);
}

extern "C" int smm_mg_upper_left(smm_mg_comm* c, const float* U_packed, const float* B, float* C_slab, int N,
                                 int ncols, int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes,
                                 void* stream) {
  SMM_RANGE("smm_mg_upper_left");
  if (int rc = check_call(c, "smm_mg_upper_left", mode, root, B, ncols)) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: bad shape or slab");
  if (int rc = check_packed("smm_mg_upper_left", N)) return rc;
  if (N == 0 || ncols == 0) return SMM_OK;
  if (nrows > 0 && (!U_packed || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: null pointer");
  if (int rc = check_ws("smm_mg_upper_left", ws, ws_bytes, smm_mg_upper_left_workspace_size(c, N, ncols, nrows, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  int cb[kMaxChunks + 1];
  const int nch = chunk_bounds(ncols, c->world, cb);
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* pack = reinterpret_cast<float*>(cur);
  uint8_t* bf = cur + (c->world > 1 ? round256(static_cast<size_t>(N) * ncols * 4) : 0);
  cur += b_side_bytes(c->world, N, ncols, mode);
  if (int rc = broadcast_blocks(c, B, N, ncols, pack, cb, nch, root, st)) return rc;
  Staged u{};  // rows [row0, row0 + nrows) of U, dense (zeros left of the diagonal)
  if (nrows > 0)
    if (int rc = expand_operand(U_packed, SMM_STRUCT_UPPER, N, row0, nrows, mode, cur, &u, st)) return rc;
  return run_blocks(c, nch, st, waits_for_blocks(c, root, mode), [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    Operand bo;
    if (int rc = block_operand(c, B, N, ncols, pack, cb, j, mode, bf, w, &bo, root)) return rc;
    Operand ao = dense_op(u.ptr, nullptr, u.ld, u.bf16);
    ao.dim = N;
    ao.row0 = row0;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ao, bo, C_slab + cb[j], ncols, nrows,
                           cb[j + 1] - cb[j], N, w, nullptr, nullptr, 0, true);
  });
}

extern "C" size_t smm_mg_toeplitz_left_workspace_size(const smm_mg_comm* c, int N, int ncols, int mode) {
  if (!c || N <= 0 || ncols <= 0) return 0;
  return b_side_bytes(c->world, N, ncols, mode);
}

extern "C" int smm_mg_toeplitz_left(smm_mg_comm* c, const float* g, const float* B, float* C_slab, int N, int ncols,
                                    int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes,
                                    void* stream) {
  SMM_RANGE("smm_mg_toeplitz_left");
  if (int rc = check_call(c, "smm_mg_toeplitz_left", mode, root, B, ncols)) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
    return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: bad shape or slab");
  if (N == 0 || ncols == 0) return SMM_OK;
  if (nrows > 0 && (!g || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: null pointer");
  if (int rc = check_ws("smm_mg_toeplitz_left", ws, ws_bytes, smm_mg_toeplitz_left_workspace_size(c, N, ncols, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  int cb[kMaxChunks + 1];
  const int nch = chunk_bounds(ncols, c->world, cb);
  float* pack = static_cast<float*>(ws);
  uint8_t* bf = static_cast<uint8_t*>(ws) + (c->world > 1 ? round256(static_cast<size_t>(N) * ncols * 4) : 0);
  if (int rc = broadcast_blocks(c, B, N, ncols, pack, cb, nch, root, st)) return rc;
  return run_blocks(c, nch, st, waits_for_blocks(c, root, mode), [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    Operand bo;
    if (int rc = block_operand(c, B, N, ncols, pack, cb, j, mode, bf, w, &bo, root)) return rc;
    return run_contraction(AKind::Toeplitz, BKind::Dense, mode, structured_op(g, N, row0), bo, C_slab + cb[j], ncols,
                           nrows, cb[j + 1] - cb[j], N, w, nullptr, nullptr, 0, true);
  });
}

namespace {
// Sandwich workspace beyond the B side: Y = A_slab S (fp32, 16-byte rows;
// plus its bf16 copy in bf16 mode), the dense expansion of S, the staged A slab.
size_t mg_sandwich_left(int N, int nrows, int mode) {
  if (nrows == 0) return 0;
  const bool bf = mode == SMM_MODE_BF16;
  return plane_bytes(nrows, N) + (bf ? bf16_plane_bytes(nrows, N) : 0) + expanded_bytes(N, N, mode) +
         staged_bytes_bound(nrows, N, mode);
}
}  // namespace

extern "C" size_t smm_mg_symm_sandwich_workspace_size(const smm_mg_comm* c, int N, int nrows, int mode) {
  if (!c || N <= 0 || nrows < 0) return 0;
  return b_side_bytes(c->world, N, N, mode) + mg_sandwich_left(N, nrows, mode);
}

extern "C" int smm_mg_symm_sandwich(smm_mg_comm* c, const float* A_slab, float* S_packed, const float* B,
                                    float* C_slab, int N, int nrows, int mode, int root, void* ws, size_t ws_bytes,
                                    void* stream) {
  SMM_RANGE("smm_mg_symm_sandwich");
  if (int rc = check_call(c, "smm_mg_symm_sandwich", mode, root, B, N)) return rc;
  if (N < 0 || nrows < 0 || nrows > N) return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: bad shape");
  if (int rc = check_packed("smm_mg_symm_sandwich", N)) return rc;
  if (N == 0) return SMM_OK;
  if (!S_packed || (nrows > 0 && (!A_slab || !C_slab)))
    return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: null pointer");
  if (int rc = check_ws("smm_mg_symm_sandwich", ws, ws_bytes, smm_mg_symm_sandwich_workspace_size(c, N, nrows, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  const bool bf = mode == SMM_MODE_BF16;
  int cb[kMaxChunks + 1];
  const int nch = chunk_bounds(N, c->world, cb);
  uint8_t* cur = static_cast<uint8_t*>(ws);
  float* pack = reinterpret_cast<float*>(cur);
  uint8_t* bfb = cur + (c->world > 1 ? round256(static_cast<size_t>(N) * N * 4) : 0);
  cur += b_side_bytes(c->world, N, N, mode);
  // S travels whole first (packed, N(N+1)/2 floats), then B in column blocks.
  if (int rc = broadcast_blocks(c, B, N, N, pack, cb, nch, root, st, S_packed, static_cast<size_t>(N) * (N + 1) / 2))
    return rc;
  float* Y = nullptr;
  __nv_bfloat16* Y_bf = nullptr;
  const int ldy = round4(N), ldy_bf = round8(N);
  if (nrows > 0) {
    // Y = A_slab S: the reference's run_graph order, (A S) first
    Y = reinterpret_cast<float*>(cur);
    cur += plane_bytes(nrows, N);
    if (bf) {
      Y_bf = reinterpret_cast<__nv_bfloat16*>(cur);
      cur += bf16_plane_bytes(nrows, N);
      if (ldy_bf != N) SMM_CUDA_TRY(cudaMemsetAsync(Y_bf, 0, bf16_plane_bytes(nrows, N), st), "zero bf16 rows");
    }
    Staged a;
    if (int rc = stage_operand(A_slab, nrows, N, mode, cur, &a, st)) return rc;
    if (c->world > 1) SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_s, 0), "wait for S");
    Staged s;  // S mirrored into a dense copy: the right operand of Y = A_slab S
    if (int rc = expand_operand(S_packed, SMM_STRUCT_SYMM, N, 0, N, mode, cur, &s, st)) return rc;
    if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, nullptr, a.ld, a.bf16),
                                 dense_op(s.ptr, nullptr, s.ld, s.bf16), bf ? nullptr : Y, ldy, nrows, N, N, st, nullptr, Y_bf,
                                 ldy_bf))
      return rc;
  }
  return run_blocks(c, nch, st, waits_for_blocks(c, root, mode), [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    Operand bo;
    if (int rc = block_operand(c, B, N, N, pack, cb, j, mode, bfb, w, &bo, root)) return rc;
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(bf ? nullptr : Y, nullptr, bf ? ldy_bf : ldy, Y_bf),
                           bo, C_slab + cb[j], N, nrows, cb[j + 1] - cb[j], N, w, nullptr, nullptr, 0, true);
  });
}
