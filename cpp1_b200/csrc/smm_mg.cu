// Multi-GPU products: one process per GPU, NCCL over NVLink / NVSwitch.
//
// A product C = X B (X the dense A, packed U, Toeplitz generator, or A S for
// the sandwich) is partitioned by output row slabs: rank g computes rows
// [r0, r1) of C.  The shared right operand B reaches every rank inside each
// call in COLUMN blocks: either broadcast from a root rank (which packs
// column block j of its B into a contiguous K x W_j buffer first), or
// all-gathered from row shares when B is sharded over the ranks (each rank
// packs its share's columns of block j; the gather concatenates the shares).
// The packs run on a pack stream, the collectives on a high-priority
// collective stream, and every rank computes
//   C_slab[:, block j] = X[r0:r1, :] B[:, block j]
// from the block as soon as it has landed, on one of several internal
// compute streams, so block j's tensor-core work overlaps the transfer of the
// blocks after it, and blocks that arrive while earlier ones still compute
// run side by side.  Every output element is written once by one full-K
// contraction (no partial sums: results identical to the single-GPU entry
// points).  In bf16 mode the blocks travel as bf16.
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

#include <fcntl.h>
#include <sched.h>
#include <sys/mman.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
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
  ncclResult_t (*allgather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
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
    api.allgather = reinterpret_cast<decltype(api.allgather)>(sym("ncclAllGather"));
    api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.broadcast &&
             api.allgather &&
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

// ---------------------------------------------------------------- copy-engine gather state
// With copy engines enabled (smm_mg_enable_copy_engines), a sharded B is
// gathered without NCCL: every rank packs its share of block j into its own
// slot of a plane buffer it registered, and its copy engines push that slot
// into the same place of every peer's plane buffer (cudaMemcpyAsync to the
// peer's buffer, mapped here through CUDA IPC).  No SM takes part in the
// transfer, so it runs beside the contractions at full speed.  Ordering
// across processes uses interprocess events -- "block j copied into rank d"
// and "rank d has finished reading its planes" -- and two host barriers per
// call (in shared memory), which make every rank's event records of a call
// precede the other ranks' waits on them.
constexpr int kMaxCeRanks = 8;
constexpr int kBarrierSeconds = 60;

struct ShmBarrier {
  std::atomic<uint32_t> arrived;
  std::atomic<uint32_t> gen;
};

struct CeState {
  uint8_t* planes = nullptr;                            // this rank's plane buffer (cudaMalloc)
  size_t bytes = 0;
  uint8_t* peer[kMaxCeRanks] = {};                      // every rank's planes, mapped here (own: planes)
  cudaStream_t xs[kMaxCeRanks] = {};                    // copy stream per destination rank
  cudaEvent_t sent[kMaxCeRanks][kMaxChunks] = {};       // recorded here: block j copied into rank d
  cudaEvent_t sent_in[kMaxCeRanks][kMaxChunks] = {};    // opened: rank s copied block j into ours
  cudaEvent_t done = nullptr;                           // recorded here: this call's readers of our planes done
  cudaEvent_t done_in[kMaxCeRanks] = {};                // opened: rank d's readers done
  cudaEvent_t xs_done[kMaxCeRanks] = {};                // local: copy stream d drained
  ShmBarrier* bar = nullptr;
  char shm_name[64] = "";
  bool owner = false;  // created the shared-memory segment (unlinks it)
};

// What each rank publishes when copy engines are enabled.
struct CeInfo {
  cudaIpcMemHandle_t mem;
  unsigned long long bytes;
  cudaIpcEventHandle_t sent[kMaxCeRanks][kMaxChunks];
  cudaIpcEventHandle_t done;
};

}  // namespace smm

// One rank's communicator: the NCCL communicator, the device it was created
// on, a high-priority stream for the collectives and one for packing the
// blocks they send, the compute streams the column blocks run on, and the
// events that order them against the caller's stream.
struct smm_mg_comm {
  ncclComm_t nc = nullptr;
  int rank = 0;
  int world = 1;
  int device = 0;
  cudaStream_t cs = nullptr;
  cudaStream_t ps = nullptr;  // packs of the blocks this rank sends
  cudaStream_t work[smm::kWork] = {};
  cudaEvent_t ev_start = nullptr;  // caller's stream: inputs ready, previous call's readers done
  cudaEvent_t ev_prep = nullptr;   // caller's stream: the left operand prepared
  cudaEvent_t ev_s = nullptr;      // collective stream: the sandwich's S arrived
  cudaEvent_t ev_cs_done = nullptr;  // collective stream: every collective (and pack) of the call done
  cudaEvent_t ev_chunk[smm::kMaxChunks] = {};
  cudaEvent_t ev_packed[smm::kMaxChunks] = {};  // pack stream: block j ready to send
  cudaEvent_t ev_done[smm::kWork] = {};
  unsigned char uid[SMM_MG_ID_BYTES] = {};
  smm::CeState* ce = nullptr;  // copy-engine gather, when enabled
};

namespace smm {
namespace {

// ---------------------------------------------------------------- partition
long long range_cost(long long n, long long a, long long b) {  // sum_{i=a}^{b-1} (n - i)
  return (b - a) * n - (b * (b - 1) - a * (a - 1)) / 2;
}

// Slab boundaries b[0] = 0 <= ... <= b[world] = n on 256-row tiles (the
// height of a CTA-pair tile: a slab of an odd number of 128-row tiles would
// end in a half-empty pair tile that costs a full one),
// minimising the largest slab's work: rows cost 1 (dense operands) or n - i
// (upper-triangular).  Binary search on the largest slab's work, then a
// greedy cut.  Slabs may be empty when n has fewer tiles than ranks.
void row_slabs(int n, int world, bool triangular, int* b) {
  constexpr int kTile = 256;
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

// Column-block boundaries of a transfer of B (ncols columns), widths
// multiples of 256 (the widest output tile).  Block count by world size
// (SMM_MG_CHUNKS overrides, 1 .. 16): 1 at world 1; 4 at world 2, where a
// rank's compute (~1.2 ms for U B 8192) outweighs the transfer and overlap
// hides it; 2 at 3-4; 1 from 5 up, where the transfer outweighs the compute
// and the blocks' collectives, competing with the contractions for SMs,
// measured slower than one transfer followed by the product (U B 8192 at 8
// GPUs, B sharded: 0.89 ms per call with 1 block, 0.91 with 2, 1.17 with 4).
// A copy-engine gather (ce) uses no SM and always takes 4 blocks.
int chunk_bounds(int ncols, int world, int* cb, bool ce = false) {
  int c = world == 1 ? 1 : world == 2 ? 4 : world <= 4 ? 2 : 1;
  if (ce && world > 1) c = 4;  // copy engines take no SM from the contractions: always overlap
  if (world > 1) {
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

// Rows of each rank's share of B when B arrives sharded by rows: ceil(K / world).
int share_rows(int K, int world) { return (K + world - 1) / world; }

// The shared right operand B of one call, in column blocks.  At world > 1
// every block travels into a contiguous plane of the workspace: from the
// root (ncclBroadcast; the root first packs the block out of its B), or,
// when B is sharded by rows, gathered from every rank's share (each rank
// packs its share's columns of the block, ncclAllGather concatenates the
// shares: rank r's rows land at r * share).  In bf16 mode the blocks travel
// as bf16 (converted before the collective: half the NVLink bytes, the same
// rounding as converting after it).  At world 1 the fp32 modes read B in
// place and bf16 converts it once.
struct BSide {
  int K = 0, ncols = 0, nch = 0;
  int cb[kMaxChunks + 1] = {};
  bool bf = false;       // blocks are bf16
  bool sharded = false;  // B arrives as row shares
  int world = 1, rank = 0, root = 0;
  int share = 0, valid = 0;  // sharded: rows per share, rows of this rank's share inside K
  int rows = 0;              // rows of a block plane
  uint8_t* planes = nullptr;
  uint8_t* send = nullptr;   // sharded: this rank's part of each block
  bool ce = false;           // sharded, gathered by copy engines into the registered planes
  int width(int j) const { return cb[j + 1] - cb[j]; }
  int ld(int j) const { return bf ? round8(width(j)) : width(j); }
  size_t esz() const { return bf ? 2 : 4; }
  size_t plane_bytes_of(int j, int r) const { return round256(static_cast<size_t>(r) * ld(j) * esz()); }
  uint8_t* plane(int j) const {
    uint8_t* p = planes;
    for (int i = 0; i < j; ++i) p += plane_bytes_of(i, rows);
    return p;
  }
  // Bytes of all block planes (rows each).
  size_t planes_bytes(int r) const {
    size_t t = 0;
    for (int j = 0; j < nch; ++j) t += plane_bytes_of(j, r);
    return t;
  }
  // This rank's slot of block j's plane (copy-engine gather): rows
  // [rank * share, rank * share + share).
  uint8_t* own_slot(int j) const { return plane(j) + static_cast<size_t>(rank) * share * ld(j) * esz(); }
  uint8_t* send_part(int j) const {
    uint8_t* p = send;
    for (int i = 0; i < j; ++i) p += plane_bytes_of(i, share);
    return p;
  }
  bool replicated = false;  // the whole B on every rank: nothing travels
  bool travels() const { return world > 1 && !replicated; }
  // Whether block j's contraction reads the caller's B in place (no wait).
  bool in_place() const { return !bf && (world == 1 || replicated || (!sharded && rank == root)); }
};

BSide make_bside(const smm_mg_comm* c, int K, int ncols, int mode, int root, void* ws) {
  BSide b;
  b.K = K;
  b.ncols = ncols;
  if (root == SMM_MG_REPLICATED) {  // one block, B (or its bf16 copy) in place on every rank
    b.replicated = true;
    b.nch = chunk_bounds(ncols, 1, b.cb);
    b.bf = mode == SMM_MODE_BF16;
    b.world = c->world;
    b.rank = c->rank;
    b.rows = K;
    b.planes = static_cast<uint8_t*>(ws);
    return b;
  }
  const bool try_ce = c->ce && root == SMM_MG_SHARDED && c->world > 1;
  b.nch = chunk_bounds(ncols, c->world, b.cb, try_ce);
  b.bf = mode == SMM_MODE_BF16;
  b.sharded = root == SMM_MG_SHARDED;
  b.world = c->world;
  b.rank = c->rank;
  b.root = b.sharded ? 0 : root;
  b.share = share_rows(K, c->world);
  b.valid = std::max(0, std::min(b.share, K - c->rank * b.share));
  b.rows = (b.sharded && c->world > 1) ? c->world * b.share : K;
  if (try_ce && c->ce->bytes >= b.planes_bytes(b.rows)) {
    b.ce = true;
    b.planes = c->ce->planes;
    return b;
  }
  if (try_ce) b.nch = chunk_bounds(ncols, c->world, b.cb, false);  // the planes do not fit: NCCL
  b.planes = static_cast<uint8_t*>(ws);
  size_t pb = 0;
  if (b.travels() || b.bf)
    for (int j = 0; j < b.nch; ++j) pb += b.plane_bytes_of(j, std::max(K, c->world * b.share));
  b.send = b.planes + pb;
  return b;
}

// Host barrier of the ranks of a copy-engine communicator (shared memory,
// generation counting); gives up after kBarrierSeconds (SMM_MG_BARRIER_MS
// sets the limit in milliseconds) with SMM_ERR_NCCL: a rank that left or
// failed is seen here, on the host, before this rank enqueues any wait on it.
int ce_barrier(CeState* e, int world, const char* who) {
  long long limit_ms = 1000LL * kBarrierSeconds;
  if (const char* env = std::getenv("SMM_MG_BARRIER_MS")) {
    const long long v = std::atoll(env);
    if (v > 0) limit_ms = v;
  }
  ShmBarrier* b = e->bar;
  const uint32_t g = b->gen.load(std::memory_order_acquire);
  if (b->arrived.fetch_add(1, std::memory_order_acq_rel) + 1 == static_cast<uint32_t>(world)) {
    b->arrived.store(0, std::memory_order_relaxed);
    b->gen.fetch_add(1, std::memory_order_release);
    return SMM_OK;
  }
  timespec t0;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (unsigned long it = 0; b->gen.load(std::memory_order_acquire) == g; ++it) {
    if ((it & 255) == 255) {
      timespec t;
      clock_gettime(CLOCK_MONOTONIC, &t);
      const long long ms = (t.tv_sec - t0.tv_sec) * 1000LL + (t.tv_nsec - t0.tv_nsec) / 1000000;
      if (ms > limit_ms)
        return set_error(SMM_ERR_NCCL, "%s: a peer rank did not reach the host barrier within %lld ms", who,
                         limit_ms);
      sched_yield();
    }
  }
  return SMM_OK;
}

// Plane buffer bytes a sharded call of this shape gathers into.
size_t ce_planes_needed(int world, int K, int ncols, int mode) {
  BSide b;
  b.K = K;
  b.ncols = ncols;
  b.nch = chunk_bounds(ncols, world, b.cb, true);
  b.bf = mode == SMM_MODE_BF16;
  b.share = share_rows(K, world);
  return b.planes_bytes(world * b.share);
}

// Workspace of the B side: the block planes (world > 1, or bf16), sized for
// the larger sharded row count, and the send parts of a sharded call.
size_t b_side_bytes(int world, int K, int ncols, int mode) {
  smm_mg_comm probe;
  probe.world = world;
  const BSide b = make_bside(&probe, K, ncols, mode, 0, nullptr);
  size_t total = 0;
  if (b.travels() || b.bf)
    for (int j = 0; j < b.nch; ++j) total += b.plane_bytes_of(j, std::max(K, world * b.share));
  if (b.travels())
    for (int j = 0; j < b.nch; ++j) total += b.plane_bytes_of(j, b.share);
  return total;
}

// Interleaved row tiles of an upper-triangular U (kMgTileRows rows each, the
// last one possibly shorter): tiles in decreasing order of work (row i costs
// n - i) each go to the rank with the least work so far (ties: the lower
// rank).  Every rank then holds long and short rows alike -- 32 tiles on 8
// ranks: {r, 15 - r, 16 + r, 31 - r} -- so the ranks' pair-tile schedules,
// and not only their work, come out even; contiguous equal-work slabs give
// the ranks with few long rows a fraction of a wave of tiles in excess.
// Writes this rank's tiles in ascending order; returns their count.
constexpr int kMgTileRows = 256;
int upper_row_tiles(int n, int world, int rank, int* tiles) {
  const int nt = (n + kMgTileRows - 1) / kMgTileRows;
  std::vector<long long> load(world, 0);
  std::vector<int> mine;
  for (int t = 0; t < nt; ++t) {  // tile t's work is larger than tile t+1's
    const long long a = static_cast<long long>(t) * kMgTileRows, e = std::min<long long>(n, a + kMgTileRows);
    const long long cost = (e - a) * n - (e * (e - 1) - a * (a - 1)) / 2;
    int g = 0;
    for (int h = 1; h < world; ++h)
      if (load[h] < load[g]) g = h;
    load[g] += cost;
    if (g == rank) mine.push_back(t);
  }
  for (size_t i = 0; i < mine.size(); ++i) tiles[i] = mine[i];
  return static_cast<int>(mine.size());
}

// Copies rows [0, rows) of column block j of src (leading dimension ncols)
// into dst (leading dimension ld(j)), fp32 or bf16; rows [rows, pad_rows) of
// dst are zeroed.
int pack_block(const BSide& b, const float* src, int rows, int pad_rows, int j, uint8_t* dst, cudaStream_t st) {
  const int w = b.width(j);
  if (rows > 0) {
    if (b.bf) {
      if (int rc = convert_block_bf16(src + b.cb[j], rows, w, b.ncols, reinterpret_cast<__nv_bfloat16*>(dst), b.ld(j),
                                      st))
        return rc;
    } else {
      pack_cols_kernel<<<148 * 4, 256, 0, st>>>(src, b.ncols, b.cb[j], rows, w, reinterpret_cast<float*>(dst));
      count_launch();
      SMM_CUDA_TRY(cudaGetLastError(), "pack column block of B");
    }
  }
  if (pad_rows > rows)
    SMM_CUDA_TRY(cudaMemsetAsync(dst + static_cast<size_t>(std::max(rows, 0)) * b.ld(j) * b.esz(), 0,
                                 static_cast<size_t>(pad_rows - std::max(rows, 0)) * b.ld(j) * b.esz(), st),
                 "zero share padding");
  return SMM_OK;
}

// Streams the copy-engine pushes of one rank go out on (SMM_MG_CE_LANES, 1 ..
// world - 1; default 1): see start_bside.
int ce_lanes(int world) {
  static const int v = [] {
    const char* e = std::getenv("SMM_MG_CE_LANES");
    return e ? std::atoi(e) : 1;
  }();
  return std::max(1, std::min(v, world - 1));
}

// Starts the B side of one call on the collective stream (ordered after the
// caller's stream): ev_chunk[j] marks block j's arrival.  The blocks this
// rank sends are packed on the pack stream, block j+1's pack overlapping
// block j's collective.  The sandwich's S_packed (s_count floats) is
// broadcast first from the root (rank 0 when B is sharded), marked by ev_s.
// At world 1, bf16 converts B on `st`.
int start_bside(smm_mg_comm* c, const BSide& b, const float* B, cudaStream_t st, float* S_packed = nullptr,
                size_t s_count = 0) {
  if (!b.travels()) {
    if (b.bf)
      return convert_block_bf16(B, b.K, b.ncols, b.ncols, reinterpret_cast<__nv_bfloat16*>(b.planes), b.ld(0), st);
    return SMM_OK;
  }
  SMM_CUDA_TRY(cudaEventRecord(c->ev_start, st), "record call start");
  SMM_CUDA_TRY(cudaStreamWaitEvent(c->cs, c->ev_start, 0), "order the collectives after the caller's stream");
  if (b.ce) {
    CeState* e = c->ce;
    const NcclApi& n = nccl();
    if (S_packed) {
      SMM_NCCL_TRY(n.broadcast(S_packed, S_packed, s_count, ncclFloat, b.root, c->nc, c->cs), "ncclBroadcast (S)");
      SMM_CUDA_TRY(cudaEventRecord(c->ev_s, c->cs), "record S arrival");
    }
    // Barrier A: every rank has recorded its end-of-call 'done' of the
    // previous call, so the waits below see this call's predecessors.
    if (int rc = ce_barrier(e, c->world, "copy-engine gather")) return rc;
    SMM_CUDA_TRY(cudaStreamWaitEvent(c->ps, c->ev_start, 0), "order the packs after the caller's stream");
    for (int j = 0; j < b.nch; ++j) {
      if (int rc = pack_block(b, B, b.valid, b.share, j, b.own_slot(j), c->ps)) return rc;
      SMM_CUDA_TRY(cudaEventRecord(c->ev_packed[j], c->ps), "record block packed");
    }
    const size_t slot_bytes_base = static_cast<size_t>(b.share) * b.esz();
    // Pushes in ring order: for each block, to ranks rank+1, rank+2, ... in
    // turn, on `lanes` streams (the copy streams of the first `lanes` of those
    // destinations), so that in step s every rank sends to rank+s and
    // receives from rank-s: one outgoing and one incoming copy per rank at a
    // time with one lane.  One stream per destination (all peers at once)
    // measured slower at 4 and 8 GPUs than at 2: a rank's pushes added up to
    // 512 GB/s with one peer, 371 with three, 314 with seven.
    const int lanes = ce_lanes(c->world);
    auto lane_of = [&](int step) { return e->xs[(c->rank + 1 + (step - 1) % lanes) % c->world]; };
    for (int d = 0; d < c->world; ++d) {
      if (d == c->rank) continue;
      // rank d's previous call has finished reading the planes we overwrite
      const int step = (d - c->rank + c->world) % c->world;
      SMM_CUDA_TRY(cudaStreamWaitEvent(lane_of(step), e->done_in[d], 0), "wait for the peer's readers");
    }
    for (int j = 0; j < b.nch; ++j) {
      const size_t off = static_cast<size_t>(b.own_slot(j) - b.planes);
      const size_t bytes = slot_bytes_base * b.ld(j);
      for (int step = 1; step < c->world; ++step) {
        const int d = (c->rank + step) % c->world;
        cudaStream_t xs = lane_of(step);
        SMM_CUDA_TRY(cudaStreamWaitEvent(xs, c->ev_packed[j], 0), "wait for the block's pack");
        SMM_CUDA_TRY(cudaMemcpyAsync(e->peer[d] + off, b.own_slot(j), bytes, cudaMemcpyDeviceToDevice, xs),
                     "copy-engine push of a share");
        SMM_CUDA_TRY(cudaEventRecord(e->sent[d][j], xs), "record block sent");
      }
    }
    // Barrier B: every rank has recorded this call's 'sent' events.
    return ce_barrier(e, c->world, "copy-engine gather");
  }
  const bool packs = b.sharded || c->rank == b.root;
  if (packs) {
    SMM_CUDA_TRY(cudaStreamWaitEvent(c->ps, c->ev_start, 0), "order the packs after the caller's stream");
    for (int j = 0; j < b.nch; ++j) {
      const int rc = b.sharded ? pack_block(b, B, b.valid, b.share, j, b.send_part(j), c->ps)
                               : pack_block(b, B, b.K, b.K, j, b.plane(j), c->ps);
      if (rc) return rc;
      SMM_CUDA_TRY(cudaEventRecord(c->ev_packed[j], c->ps), "record block packed");
    }
  }
  const NcclApi& n = nccl();
  if (S_packed) {
    SMM_NCCL_TRY(n.broadcast(S_packed, S_packed, s_count, ncclFloat, b.root, c->nc, c->cs), "ncclBroadcast (S)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_s, c->cs), "record S arrival");
  }
  const ncclDataType_t ty = b.bf ? ncclBfloat16 : ncclFloat;
  for (int j = 0; j < b.nch; ++j) {
    if (packs) SMM_CUDA_TRY(cudaStreamWaitEvent(c->cs, c->ev_packed[j], 0), "wait for the block's pack");
    if (b.sharded)
      SMM_NCCL_TRY(n.allgather(b.send_part(j), b.plane(j), static_cast<size_t>(b.share) * b.ld(j), ty, c->nc, c->cs),
                   "ncclAllGather (column block of B)");
    else
      SMM_NCCL_TRY(n.broadcast(b.plane(j), b.plane(j), static_cast<size_t>(b.K) * b.ld(j), ty, b.root, c->nc, c->cs),
                   "ncclBroadcast (column block of B)");
    SMM_CUDA_TRY(cudaEventRecord(c->ev_chunk[j], c->cs), "record block arrival");
  }
  return SMM_OK;
}

// Runs block(j, stream) for every column block: at world 1 the single block
// on the caller's stream; else block j on compute stream j % kWork once the
// left operand is prepared (ev_prep, recorded on the caller's stream) and,
// unless it reads B in place, the block has landed; the caller's stream then
// waits for all of them.
template <typename F>
int run_blocks(smm_mg_comm* c, const BSide& b, cudaStream_t st, F&& block) {
  if (!b.travels()) return block(0, st);
  SMM_CUDA_TRY(cudaEventRecord(c->ev_prep, st), "record operand preparation");
  const int used = std::min(b.nch, kWork);
  for (int w = 0; w < used; ++w) SMM_CUDA_TRY(cudaStreamWaitEvent(c->work[w], c->ev_prep, 0), "fork");
  for (int j = 0; j < b.nch; ++j) {
    cudaStream_t w = c->work[j % kWork];
    if (b.ce) {
      SMM_CUDA_TRY(cudaStreamWaitEvent(w, c->ev_packed[j], 0), "wait for this rank's slot");
      for (int s = 0; s < c->world; ++s)
        if (s != c->rank) SMM_CUDA_TRY(cudaStreamWaitEvent(w, c->ce->sent_in[s][j], 0), "wait for a peer's share");
    } else if (!b.in_place()) {
      SMM_CUDA_TRY(cudaStreamWaitEvent(w, c->ev_chunk[j], 0), "wait for block arrival");
    }
    if (int rc = block(j, w)) return rc;
  }
  for (int w = 0; w < used; ++w) {
    SMM_CUDA_TRY(cudaEventRecord(c->ev_done[w], c->work[w]), "record block done");
    SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_done[w], 0), "join");
  }
  if (b.ce) {
    // our pushes have read our slots; then our planes are fully read
    for (int d = 0; d < c->world; ++d) {
      if (d == c->rank) continue;
      SMM_CUDA_TRY(cudaEventRecord(c->ce->xs_done[d], c->ce->xs[d]), "record pushes done");
      SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ce->xs_done[d], 0), "join the pushes");
    }
    SMM_CUDA_TRY(cudaEventRecord(c->ce->done, st), "record planes read");
  }
  // The caller's stream also waits for the collectives (and, through them,
  // the packs that read B): the root computing from B in place does not wait
  // for its own sends, and the next call's packs must not overwrite a block
  // still being sent.
  SMM_CUDA_TRY(cudaEventRecord(c->ev_cs_done, c->cs), "record collectives done");
  SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_cs_done, 0), "join the collectives");
  return SMM_OK;
}

// Tiles of the column-block products.  With more than one rank the blocks'
// products run side by side on the compute streams, so each takes 256 x 256
// pair tiles (the fastest per flop) instead of the narrower or K-split tiles
// a launch that had the GPU to itself would take: at 8 GPUs the first slab
// of U B 8192 (512 rows, K ~ 8000) ran as 512 single-CTA split tiles, about
// four waves, against one wave of 64 pair tiles.  SMM_MG_TILES=auto restores
// the single-launch choice.
TilePolicy block_tiles(const smm_mg_comm* c) {
  static const bool forced_auto = [] {
    const char* e = std::getenv("SMM_MG_TILES");
    return e && std::strcmp(e, "auto") == 0;
  }();
  return (c->world > 1 && !forced_auto) ? TilePolicy::WidePairs : TilePolicy::Auto;
}

// The B operand of column block j (K x W_j): the caller's B in place, or the
// block's plane (fp32 or bf16).
Operand block_operand(const BSide& b, const float* B, int j) {
  if (b.in_place()) return dense_op(B + b.cb[j], nullptr, b.ncols);
  if (b.bf) return dense_op(nullptr, nullptr, b.ld(j), reinterpret_cast<const __nv_bfloat16*>(b.plane(j)));
  return dense_op(reinterpret_cast<const float*>(b.plane(j)), nullptr, b.ld(j));
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
// Frees the copy-engine state.  `wait_peers`: first close this rank's
// mappings of the peers' planes and wait (host barrier) until every rank has
// closed its mappings of ours before freeing them (a normal destroy; an abort
// does not wait for peers).
void ce_release(smm_mg_comm* c, bool wait_peers) {
  CeState* e = c->ce;
  if (!e) return;
  for (auto& x : e->xs)
    if (x) cudaStreamSynchronize(x);
  for (int s = 0; s < kMaxCeRanks; ++s) {
    if (s != c->rank && e->peer[s]) cudaIpcCloseMemHandle(e->peer[s]);
    e->peer[s] = nullptr;
    for (auto& ev : e->sent_in[s])
      if (ev) cudaEventDestroy(ev);
    if (e->done_in[s]) cudaEventDestroy(e->done_in[s]);
  }
  if (wait_peers && e->bar) ce_barrier(e, c->world, "copy-engine teardown");
  for (auto& row : e->sent)
    for (auto& ev : row)
      if (ev) cudaEventDestroy(ev);
  if (e->done) cudaEventDestroy(e->done);
  for (auto& ev : e->xs_done)
    if (ev) cudaEventDestroy(ev);
  for (auto& x : e->xs)
    if (x) cudaStreamDestroy(x);
  if (e->planes) cudaFree(e->planes);
  if (e->bar) munmap(e->bar, sizeof(ShmBarrier));
  if (e->owner) shm_unlink(e->shm_name);
  delete e;
  c->ce = nullptr;
}

void release(smm_mg_comm* c) {
  ce_release(c, false);
  if (c->cs) cudaStreamDestroy(c->cs);
  if (c->ps) cudaStreamDestroy(c->ps);
  for (auto& w : c->work)
    if (w) cudaStreamDestroy(w);
  for (cudaEvent_t e : {c->ev_start, c->ev_prep, c->ev_s, c->ev_cs_done})
    if (e) cudaEventDestroy(e);
  for (auto& e : c->ev_chunk)
    if (e) cudaEventDestroy(e);
  for (auto& e : c->ev_packed)
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
      cudaStreamCreateWithPriority(&c->cs, cudaStreamNonBlocking, hi) != cudaSuccess ||
      cudaStreamCreateWithPriority(&c->ps, cudaStreamNonBlocking, hi) != cudaSuccess)
    return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: collective streams"));
  for (auto& w : c->work)
    if (cudaStreamCreateWithFlags(&w, cudaStreamNonBlocking) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: compute stream"));
  for (cudaEvent_t* e : {&c->ev_start, &c->ev_prep, &c->ev_s, &c->ev_cs_done})
    if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  for (auto& e : c->ev_chunk)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
      return fail(set_error(SMM_ERR_CUDA, "smm_mg_comm_init: event"));
  for (auto& e : c->ev_packed)
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
    std::memcpy(c->uid, id, sizeof(c->uid));
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
  if (c->ps) cudaStreamSynchronize(c->ps);
  for (auto& w : c->work)
    if (w) cudaStreamSynchronize(w);
  ce_release(c, true);
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

// ---------------------------------------------------------------- copy-engine gather
namespace {
int ce_enable(smm_mg_comm* c, size_t plane_bytes) {
  auto* e = new CeState();
  c->ce = e;
  const int world = c->world, rank = c->rank;
  // Host barrier segment, named by the communicator's unique id: rank 0
  // creates it before the exchange below, the others open it after.
  unsigned long long h0 = 0, h1 = 0;
  std::memcpy(&h0, c->uid, 8);
  std::memcpy(&h1, c->uid + 8, 8);
  snprintf(e->shm_name, sizeof(e->shm_name), "/smm_mg_%016llx%016llx", h0, h1);
  auto map_bar = [&](bool create) -> int {
    int fd = create ? shm_open(e->shm_name, O_CREAT | O_EXCL | O_RDWR, 0600) : shm_open(e->shm_name, O_RDWR, 0);
    if (fd < 0) return set_error(SMM_ERR_CUDA, "copy engines: shm_open(%s) failed", e->shm_name);
    if (create && ftruncate(fd, sizeof(ShmBarrier)) != 0) {
      close(fd);
      return set_error(SMM_ERR_CUDA, "copy engines: ftruncate of the barrier segment failed");
    }
    void* p = mmap(nullptr, sizeof(ShmBarrier), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return set_error(SMM_ERR_CUDA, "copy engines: mmap of the barrier segment failed");
    e->bar = static_cast<ShmBarrier*>(p);
    e->owner = create;
    return SMM_OK;
  };
  // Local set-up.  A failure here still takes part in the exchange (with a
  // zero byte count), so that every rank returns the error instead of
  // leaving the others in the collective.
  CeInfo info;
  std::memset(&info, 0, sizeof(info));
  auto local = [&]() -> int {
    if (rank == 0) {
      shm_unlink(e->shm_name);  // a stale segment of a crashed run with the same id
      if (int rc = map_bar(true)) return rc;
    }
    SMM_CUDA_TRY(cudaMalloc(&e->planes, plane_bytes), "copy engines: plane buffer");
    e->bytes = plane_bytes;
    SMM_CUDA_TRY(cudaIpcGetMemHandle(&info.mem, e->planes), "cudaIpcGetMemHandle");
    int lo = 0, hi = 0;
    SMM_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&lo, &hi), "stream priorities");
    for (int d = 0; d < world; ++d) {
      if (d == rank) continue;
      SMM_CUDA_TRY(cudaStreamCreateWithPriority(&e->xs[d], cudaStreamNonBlocking, hi), "copy stream");
      SMM_CUDA_TRY(cudaEventCreateWithFlags(&e->xs_done[d], cudaEventDisableTiming), "event");
      for (int j = 0; j < kMaxChunks; ++j) {
        SMM_CUDA_TRY(cudaEventCreateWithFlags(&e->sent[d][j], cudaEventDisableTiming | cudaEventInterprocess),
                     "interprocess event");
        SMM_CUDA_TRY(cudaIpcGetEventHandle(&info.sent[d][j], e->sent[d][j]), "cudaIpcGetEventHandle");
      }
    }
    SMM_CUDA_TRY(cudaEventCreateWithFlags(&e->done, cudaEventDisableTiming | cudaEventInterprocess),
                 "interprocess event");
    SMM_CUDA_TRY(cudaIpcGetEventHandle(&info.done, e->done), "cudaIpcGetEventHandle");
    info.bytes = plane_bytes;
    return SMM_OK;
  };
  const int local_rc = local();
  if (local_rc) info.bytes = 0;
  // Exchange (one NCCL all-gather of the records; set-up only).
  CeInfo* dev = nullptr;
  SMM_CUDA_TRY(cudaMalloc(&dev, sizeof(CeInfo) * world), "exchange buffer");
  std::vector<CeInfo> all(world);
  int rc = SMM_OK;
  if (cudaMemcpy(dev + rank, &info, sizeof(CeInfo), cudaMemcpyHostToDevice) != cudaSuccess) {
    rc = set_error(SMM_ERR_CUDA, "copy engines: exchange copy");
  } else {
    ncclResult_t r = nccl().allgather(dev + rank, dev, sizeof(CeInfo), ncclUint8, c->nc, c->cs);
    if (r != ncclSuccess)
      rc = nccl_fail(r, "ncclAllGather (copy-engine exchange)");
    else if (cudaStreamSynchronize(c->cs) != cudaSuccess ||
             cudaMemcpy(all.data(), dev, sizeof(CeInfo) * world, cudaMemcpyDeviceToHost) != cudaSuccess)
      rc = set_error(SMM_ERR_CUDA, "copy engines: exchange");
  }
  cudaFree(dev);
  if (local_rc) return local_rc;
  if (rc) return rc;
  for (int s = 0; s < world; ++s)
    if (all[s].bytes != plane_bytes)
      return set_error(SMM_ERR_INVALID,
                       "smm_mg_enable_copy_engines: rank %d set up %llu plane bytes (0: its set-up failed), this "
                       "rank %zu",
                       s, all[s].bytes, plane_bytes);
  e->peer[rank] = e->planes;
  for (int s = 0; s < world; ++s) {
    if (s == rank) continue;
    void* p = nullptr;
    SMM_CUDA_TRY(cudaIpcOpenMemHandle(&p, all[s].mem, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    e->peer[s] = static_cast<uint8_t*>(p);
    for (int j = 0; j < kMaxChunks; ++j)
      SMM_CUDA_TRY(cudaIpcOpenEventHandle(&e->sent_in[s][j], all[s].sent[rank][j]), "cudaIpcOpenEventHandle");
    SMM_CUDA_TRY(cudaIpcOpenEventHandle(&e->done_in[s], all[s].done), "cudaIpcOpenEventHandle");
  }
  if (rank != 0)
    if (int rc2 = map_bar(false)) return rc2;
  return ce_barrier(e, world, "smm_mg_enable_copy_engines");
}
}  // namespace

extern "C" size_t smm_mg_plane_bytes(const smm_mg_comm* c, int K, int ncols, int mode) {
  if (!c || K <= 0 || ncols <= 0 || !valid_mode(mode) || c->world < 2) return 0;
  return ce_planes_needed(c->world, K, ncols, mode);
}

extern "C" int smm_mg_enable_copy_engines(smm_mg_comm* c, size_t plane_bytes) {
  SMM_RANGE("smm_mg_enable_copy_engines");
  if (int rc = check_comm(c, "smm_mg_enable_copy_engines")) return rc;
  if (c->world == 1) return SMM_OK;  // nothing travels
  if (c->world > kMaxCeRanks)
    return set_error(SMM_ERR_UNSUPPORTED, "smm_mg_enable_copy_engines: at most %d ranks", kMaxCeRanks);
  if (plane_bytes == 0) return set_error(SMM_ERR_INVALID, "smm_mg_enable_copy_engines: zero plane bytes");
  if (c->ce) {
    for (auto& w : c->work) cudaStreamSynchronize(w);
    ce_release(c, true);
  }
  const int rc = ce_enable(c, plane_bytes);
  if (rc) ce_release(c, false);
  return rc;
}

extern "C" int smm_mg_copy_engines_enabled(const smm_mg_comm* c) { return c && c->ce ? 1 : 0; }

extern "C" int smm_mg_upper_row_tiles(int N, int world, int rank, int* tiles, int max_tiles, int* count) {
  if (N < 0 || world < 1 || rank < 0 || rank >= world || max_tiles < 0 || (!tiles && max_tiles > 0) || !count)
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_row_tiles: bad arguments");
  const int nt = (N + kMgTileRows - 1) / kMgTileRows;
  std::vector<int> all(static_cast<size_t>(nt) + 1);
  const int k = upper_row_tiles(N, world, rank, all.data());
  if (k > max_tiles) return set_error(SMM_ERR_INVALID, "smm_mg_upper_row_tiles: %d tiles, room for %d", k, max_tiles);
  for (int i = 0; i < k; ++i) tiles[i] = all[i];
  *count = k;
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

extern "C" int smm_mg_gather_chunks(int ncols, int world, int* bounds) {
  if (ncols < 0 || world < 1 || !bounds) return set_error(SMM_ERR_INVALID, "smm_mg_gather_chunks: bad arguments");
  return chunk_bounds(ncols, world, bounds, true);
}

namespace {
// Validation shared by the products: B (K x ncols) is the root's whole B,
// or with root SMM_MG_SHARDED this rank's share (rows [rank * s, rank * s +
// valid) of B, s = smm_mg_share_rows(K, world)); either with 16-byte aligned
// rows when it holds any.
int check_call(const smm_mg_comm* c, const char* who, int mode, int root, const float* B, int K, int ncols) {
  if (int rc = check_comm(c, who)) return rc;
  if (root != SMM_MG_SHARDED && root != SMM_MG_REPLICATED && (root < 0 || root >= c->world))
    return set_error(SMM_ERR_INVALID, "%s: root %d of %d", who, root, c->world);
  if (!valid_mode(mode)) return set_error(SMM_ERR_INVALID, "%s: unknown mode %d", who, mode);
  const bool holds = root == SMM_MG_SHARDED      ? (K - c->rank * share_rows(K, c->world) > 0)
                     : root == SMM_MG_REPLICATED ? true
                                                 : c->rank == root;
  if (holds && K > 0 && ncols > 0 && (!B || !aligned_rows(B, ncols)))
    return set_error(SMM_ERR_INVALID, "%s: this rank's B must be non-null with 16-byte aligned rows", who);
  return SMM_OK;
}
}  // namespace

extern "C" int smm_mg_share_rows(int K, int world) {
  if (K < 0 || world < 1) return set_error(SMM_ERR_INVALID, "smm_mg_share_rows: bad arguments");
  return share_rows(K, world);
}

// ---------------------------------------------------------------- products
extern "C" size_t smm_mg_gemm_workspace_size(const smm_mg_comm* c, int nrows, int N, int K, int mode) {
  if (!c || nrows < 0 || N <= 0 || K <= 0) return 0;
  return b_side_bytes(c->world, K, N, mode) + (nrows ? staged_bytes_bound(nrows, K, mode) : 0);
}

extern "C" int smm_mg_gemm(smm_mg_comm* c, const float* A_slab, const float* B, float* C_slab, int nrows, int N,
                           int K, int mode, int root, void* ws, size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_gemm");
  if (int rc = check_call(c, "smm_mg_gemm", mode, root, B, K, N)) return rc;
  if (nrows < 0 || N < 0 || K < 0) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: negative shape");
  if (N == 0 || K == 0) return SMM_OK;
  if (nrows > 0 && (!A_slab || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_gemm: null pointer");
  if (int rc = check_ws("smm_mg_gemm", ws, ws_bytes, smm_mg_gemm_workspace_size(c, nrows, N, K, mode))) return rc;
  cudaStream_t st = as_stream(stream);
  const BSide b = make_bside(c, K, N, mode, root, ws);
  uint8_t* cur = static_cast<uint8_t*>(ws) + b_side_bytes(c->world, K, N, mode);
  if (int rc = start_bside(c, b, B, st)) return rc;
  Staged a{};
  if (nrows > 0)
    if (int rc = stage_operand(A_slab, nrows, K, mode, cur, &a, st)) return rc;
  return run_blocks(c, b, st, [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, nullptr, a.ld, a.bf16),
                           block_operand(b, B, j), C_slab + b.cb[j], N, nrows, b.width(j), K, w, nullptr, nullptr, 0,
                           block_tiles(c));
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
  if (int rc = check_call(c, "smm_mg_upper_left", mode, root, B, N, ncols)) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: bad shape or slab");
  if (int rc = check_packed("smm_mg_upper_left", N)) return rc;
  if (N == 0 || ncols == 0) return SMM_OK;
  if (nrows > 0 && (!U_packed || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_upper_left: null pointer");
  if (int rc = check_ws("smm_mg_upper_left", ws, ws_bytes, smm_mg_upper_left_workspace_size(c, N, ncols, nrows, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  const BSide b = make_bside(c, N, ncols, mode, root, ws);
  uint8_t* cur = static_cast<uint8_t*>(ws) + b_side_bytes(c->world, N, ncols, mode);
  if (int rc = start_bside(c, b, B, st)) return rc;
  Staged u{};  // rows [row0, row0 + nrows) of U, dense (zeros left of the diagonal)
  if (nrows > 0)
    if (int rc = expand_operand(U_packed, SMM_STRUCT_UPPER, N, row0, nrows, mode, cur, &u, st)) return rc;
  return run_blocks(c, b, st, [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    Operand ao = dense_op(u.ptr, nullptr, u.ld, u.bf16);
    ao.dim = N;
    ao.row0 = row0;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ao, block_operand(b, B, j), C_slab + b.cb[j],
                           ncols, nrows, b.width(j), N, w, nullptr, nullptr, 0, block_tiles(c));
  });
}

extern "C" size_t smm_mg_upper_left_tiles_workspace_size(const smm_mg_comm* c, int N, int ncols, int ntiles,
                                                        int mode) {
  if (!c || N <= 0 || ncols <= 0 || ntiles < 0) return 0;
  return b_side_bytes(c->world, N, ncols, mode) +
         (ntiles ? expanded_bytes(std::min(N, ntiles * kMgTileRows), N, mode) : 0);
}

extern "C" int smm_mg_upper_left_tiles(smm_mg_comm* c, const float* U_packed, const float* B, float* C_rows, int N,
                                       int ncols, const int* tiles, int ntiles, int mode, int root, void* ws,
                                       size_t ws_bytes, void* stream) {
  SMM_RANGE("smm_mg_upper_left_tiles");
  if (int rc = check_call(c, "smm_mg_upper_left_tiles", mode, root, B, N, ncols)) return rc;
  if (N < 0 || ncols < 0 || ntiles < 0 || ntiles > kMaxMappedTiles)
    return set_error(SMM_ERR_INVALID, "smm_mg_upper_left_tiles: bad shape or tile count %d (at most %d)", ntiles,
                     kMaxMappedTiles);
  if (int rc = check_packed("smm_mg_upper_left_tiles", N)) return rc;
  const int nt = (N + kMgTileRows - 1) / kMgTileRows;
  int rows = 0;
  int row0[kMaxMappedTiles];
  for (int i = 0; i < ntiles; ++i) {
    if (!tiles || tiles[i] < 0 || tiles[i] >= nt || (i > 0 && tiles[i] <= tiles[i - 1]))
      return set_error(SMM_ERR_INVALID, "smm_mg_upper_left_tiles: tiles must be ascending row tiles of U (0 .. %d)",
                       nt - 1);
    row0[i] = tiles[i] * kMgTileRows;
    rows += std::min(kMgTileRows, N - row0[i]);
  }
  if (N == 0 || ncols == 0) return SMM_OK;
  if (rows > 0 && (!U_packed || !C_rows)) return set_error(SMM_ERR_INVALID, "smm_mg_upper_left_tiles: null pointer");
  if (int rc = check_ws("smm_mg_upper_left_tiles", ws, ws_bytes,
                        smm_mg_upper_left_tiles_workspace_size(c, N, ncols, ntiles, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  const BSide b = make_bside(c, N, ncols, mode, root, ws);
  uint8_t* cur = static_cast<uint8_t*>(ws) + b_side_bytes(c->world, N, ncols, mode);
  if (int rc = start_bside(c, b, B, st)) return rc;
  // The tiles' rows of U, dense (zeros left of the diagonal), stacked in
  // order by one expansion launch (separate 256-row launches cost ~8 us
  // each: 23 of them added ~0.15 ms to a rank's call).
  Staged u{};
  if (rows > 0)
    if (int rc = expand_operand_tiles(U_packed, SMM_STRUCT_UPPER, N, row0, ntiles, kMgTileRows, rows, mode, cur, &u,
                                      st))
      return rc;
  return run_blocks(c, b, st, [&](int j, cudaStream_t w) -> int {
    if (rows == 0) return SMM_OK;
    Operand ao = dense_op(u.ptr, nullptr, u.ld, u.bf16);
    ao.dim = N;
    ao.tile_rows = kMgTileRows;
    ao.tile_row0 = row0;
    ao.ntiles = ntiles;
    return run_contraction(AKind::UpperDense, BKind::Dense, mode, ao, block_operand(b, B, j), C_rows + b.cb[j],
                           ncols, rows, b.width(j), N, w, nullptr, nullptr, 0, block_tiles(c));
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
  if (int rc = check_call(c, "smm_mg_toeplitz_left", mode, root, B, N, ncols)) return rc;
  if (N < 0 || ncols < 0 || row0 < 0 || nrows < 0 || row0 + nrows > N)
    return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: bad shape or slab");
  if (N == 0 || ncols == 0) return SMM_OK;
  if (nrows > 0 && (!g || !C_slab)) return set_error(SMM_ERR_INVALID, "smm_mg_toeplitz_left: null pointer");
  if (int rc = check_ws("smm_mg_toeplitz_left", ws, ws_bytes, smm_mg_toeplitz_left_workspace_size(c, N, ncols, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  const BSide b = make_bside(c, N, ncols, mode, root, ws);
  if (int rc = start_bside(c, b, B, st)) return rc;
  return run_blocks(c, b, st, [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    return run_contraction(AKind::Toeplitz, BKind::Dense, mode, structured_op(g, N, row0), block_operand(b, B, j),
                           C_slab + b.cb[j], ncols, nrows, b.width(j), N, w, nullptr, nullptr, 0, block_tiles(c));
  });
}

namespace {
// Sandwich workspace beyond the B side: Y = A_slab S (bf16 in bf16 mode,
// else fp32; 16-byte rows), the dense expansion of S, the staged A slab.
size_t mg_sandwich_left(int N, int nrows, int mode) {
  if (nrows == 0) return 0;
  const bool bf = mode == SMM_MODE_BF16;
  return (bf ? bf16_plane_bytes(nrows, N) : plane_bytes(nrows, N)) + expanded_bytes(N, N, mode) +
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
  if (int rc = check_call(c, "smm_mg_symm_sandwich", mode, root, B, N, N)) return rc;
  if (N < 0 || nrows < 0 || nrows > N) return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: bad shape");
  if (int rc = check_packed("smm_mg_symm_sandwich", N)) return rc;
  if (N == 0) return SMM_OK;
  if (!S_packed || (nrows > 0 && (!A_slab || !C_slab)))
    return set_error(SMM_ERR_INVALID, "smm_mg_symm_sandwich: null pointer");
  if (int rc = check_ws("smm_mg_symm_sandwich", ws, ws_bytes, smm_mg_symm_sandwich_workspace_size(c, N, nrows, mode)))
    return rc;
  cudaStream_t st = as_stream(stream);
  const bool bf = mode == SMM_MODE_BF16;
  const BSide b = make_bside(c, N, N, mode, root, ws);
  uint8_t* cur = static_cast<uint8_t*>(ws) + b_side_bytes(c->world, N, N, mode);
  // S travels whole first (packed, N(N+1)/2 floats, from the root; rank 0
  // when B is sharded), then B in column blocks.
  if (int rc = start_bside(c, b, B, st, S_packed, static_cast<size_t>(N) * (N + 1) / 2)) return rc;
  float* Y = nullptr;
  __nv_bfloat16* Y_bf = nullptr;
  const int ldy = bf ? round8(N) : round4(N);
  if (nrows > 0) {
    // Y = A_slab S: the reference's run_graph order, (A S) first; in bf16
    // mode only Y's bf16 copy is written (the second product's operand)
    if (bf) {
      Y_bf = reinterpret_cast<__nv_bfloat16*>(cur);
      cur += bf16_plane_bytes(nrows, N);
      if (ldy != N) SMM_CUDA_TRY(cudaMemsetAsync(Y_bf, 0, bf16_plane_bytes(nrows, N), st), "zero bf16 rows");
    } else {
      Y = reinterpret_cast<float*>(cur);
      cur += plane_bytes(nrows, N);
    }
    Staged a;
    if (int rc = stage_operand(A_slab, nrows, N, mode, cur, &a, st)) return rc;
    if (c->world > 1) SMM_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_s, 0), "wait for S");
    Staged s;  // S mirrored into a dense copy: the right operand of Y = A_slab S
    if (int rc = expand_operand(S_packed, SMM_STRUCT_SYMM, N, 0, N, mode, cur, &s, st)) return rc;
    if (int rc = run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(a.ptr, nullptr, a.ld, a.bf16),
                                 dense_op(s.ptr, nullptr, s.ld, s.bf16), Y, ldy, nrows, N, N, st, nullptr, Y_bf,
                                 ldy))
      return rc;
  }
  return run_blocks(c, b, st, [&](int j, cudaStream_t w) -> int {
    if (nrows == 0) return SMM_OK;
    return run_contraction(AKind::Dense, BKind::Dense, mode, dense_op(Y, nullptr, ldy, Y_bf), block_operand(b, B, j),
                           C_slab + b.cb[j], N, nrows, b.width(j), N, w, nullptr, nullptr, 0, block_tiles(c));
  });
}
