// The tcgen05 contraction engine shared by every tensor-core operation of the
// library: C(M x N) = Aop(M x K) * B(K x N), fp32 row-major C, accumulator in
// tensor memory.
//
// Tile: 128 x BN output per CTA (BN = 64, 128 or 256), K-blocks of 16 fp32
// (64 bytes) per pipeline stage, STAGES stages in shared memory.
//
// Operand staging per stage:
//   A (K-major, 128 rows x 64 B, 64-byte swizzle):
//     AKind::Dense       TMA tile load of a row-major A
//     AKind::UpperPacked built by the transform warps from packed-upper
//                        storage (zeros below the diagonal; k-blocks left of
//                        the row tile's diagonal are never visited)
//     AKind::Toeplitz    built from the 2N-1 generator: row r of the tile is
//                        a contiguous generator window
//     AKind::SymmPacked  built from packed-upper storage, mirrored below the
//                        diagonal
//   B (MN-major, BN columns x 16 k-rows): TMA tile loads of a row-major B,
//     32 columns (128 B) per box, 128-byte swizzle with 32-byte atoms (the
//     only swizzle kind::tf32 accepts for an MN-major operand; with the plain
//     128-byte swizzle the MMA produces nothing).
//
// 3xTF32 (SPLIT3): the transform warps write lo = x - tf32(x) planes of both
// operands next to the raw tiles, and the MMA issuer runs three MMAs per
// k-step: hi*hi + hi*lo + lo*hi.  The raw fp32 tile serves as the hi operand
// (kind::tf32 reads the upper 19 bits of each element).
//
// Warp roles (192 threads):
//   warp 0     TMA producer (one lane)
//   warp 1     TMEM allocator + MMA issuer (one lane)
//   warps 2-5  transform (lo planes, structured A tiles), then epilogue
//              (TMEM -> registers -> global C)
//
// Every wait is bounded (WaitCtx): on expiry the kernel records
// kDevErrTimeout in the status word, the other roles stop waiting, in-flight
// copies/MMAs are drained (bounded), TMEM is freed and the CTA exits.
#pragma once
#include "smm_device.cuh"

namespace smm {

enum class AKind : int { Dense = 0, UpperPacked = 1, Toeplitz = 2, SymmPacked = 3, UpperDense = 4 };
// Right operand: a dense row-major matrix loaded by TMA, or a packed
// upper-triangular / symmetric matrix built on chip by the transform warps.
enum class BKind : int { Dense = 0, UpperPacked = 1, SymmPacked = 2 };

struct UmmaParams {
  int M, N, K;             // C is M x N; reduction length K
  float* C;                // row-major, leading dimension ldc
  int ldc;
  const float* a_src;      // packed U / generator / packed S (structured A kinds)
  int a_dim;               // order of the structured matrix
  int a_row0;              // row of the structured matrix that output row 0 maps to
  const float* b_src;      // packed U / packed S (structured B kinds)
  int b_dim;               // order of the structured right operand
  int row_tiles;           // ceil(M / 128)
  int col_tiles;           // ceil(N / BN)
  uint32_t* status;        // device status word (sticky error bits)
  unsigned long long wait_limit_ns;
  uint32_t* trace;         // optional diagnostic record of CTA (0,0); null in normal use
};

// Slots of the diagnostic record (UmmaParams::trace, 64 words).
enum : int {
  kTrTmem = 0, kTrNumKb = 1, kTrA = 2 /*8 words*/, kTrB = 10 /*8 words*/, kTrAccOk = 18,
  kTrAcc = 19 /*16 words*/, kTrMmas = 35, kTrDescA = 36 /*2 words*/, kTrDescB = 38 /*2*/, kTrIdesc = 40,
  kTrEpiDone = 41, kTrWords = 64
};

constexpr int kBM = 128;
constexpr int kBK = 16;                   // fp32 elements per k-block (64 bytes)
constexpr int kThreads = 192;
constexpr int kATileBytes = kBM * kBK * 4;  // 8 KiB

template <int BN>
struct TileGeom {
  static constexpr int kBTileBytes = BN * kBK * 4;  // BN/32 boxes of 16 rows x 128 B
  static constexpr int kBChunkBytes = 16 * 128;     // one 32-column box
};

template <int BN, bool SPLIT3>
__host__ __device__ constexpr int stage_bytes() {
  return (SPLIT3 ? 2 : 1) * (kATileBytes + TileGeom<BN>::kBTileBytes);
}

// 3xTF32 accumulates in chunks of kChunk k-blocks: the tensor core's fp32
// accumulation truncates on every update, so with same-sign data its error
// grows with the number of updates into one accumulator.  Each chunk goes
// to one of two ping-pong accumulators (overwritten at chunk start) and the
// transform warps fold finished chunks into a third TMEM region with
// round-to-nearest fp32 adds, bounding the truncation bias to
// 3 * kChunk * 2 updates whatever K is.
constexpr int kChunk = 8;

template <int BN, bool SPLIT3>
__host__ __device__ constexpr uint32_t tmem_cols() {
  // SPLIT3: acc0 [0,BN), acc1 [BN,2BN), running sum [2BN,3BN)
  return SPLIT3 ? (3 * BN <= 256 ? 256u : 512u) : (BN < 32 ? 32u : static_cast<uint32_t>(BN));
}

template <int BN, bool SPLIT3, int STAGES>
__host__ __device__ constexpr int umma_smem_bytes() {
  return 1024 /*alignment slack*/ + STAGES * stage_bytes<BN, SPLIT3>() + 256 /*barriers etc*/;
}

__device__ __forceinline__ long long packed_idx(long long i, long long j, long long n) {
  return i * n - i * (i - 1) / 2 + (j - i);
}

// Value of the structured left operand at (row gr, column k); zero outside
// the n x n matrix.
template <AKind AK>
__device__ __forceinline__ float a_value(const float* __restrict__ src, int n, int gr, int k) {
  if (gr >= n || k >= n) return 0.0f;
  if constexpr (AK == AKind::UpperPacked) {
    return k >= gr ? __ldg(src + packed_idx(gr, k, n)) : 0.0f;
  } else if constexpr (AK == AKind::Toeplitz) {
    return __ldg(src + (n - 1 + k - gr));
  } else {  // SymmPacked
    return k >= gr ? __ldg(src + packed_idx(gr, k, n)) : __ldg(src + packed_idx(k, gr, n));
  }
}

// The 16 values one transform thread contributes to a structured A stage
// tile (rows m0.., columns k0..k0+15), gathered into registers so all 16
// loads are in flight together (the tile is rebuilt every stage, so load
// latency, not bandwidth, bounds this producer).
//   lanes along k (16 lanes per row, two rows per warp instruction): rows
//     tw*32 + 2*it + lane/16, column lane%16 — coalesced along a packed row
//     or a generator window;
//   lanes along rows (symmetric tiles wholly below the diagonal, whose
//     elements are the mirror S[k][row]): row tw*32 + lane, column it —
//     coalesced along packed row k.
template <AKind AK>
__device__ __forceinline__ bool a_rows_mapping(int g_first, int k0) {
  return AK == AKind::SymmPacked && k0 + kBK <= g_first;
}

template <AKind AK>
__device__ __forceinline__ void a_gather(float (&v)[16], const UmmaParams& p, int g_first, int k0, int tw,
                                         int lane) {
  if (a_rows_mapping<AK>(g_first, k0)) {
    const int gr = g_first + tw * 32 + lane;
#pragma unroll
    for (int it = 0; it < 16; ++it) v[it] = a_value<AK>(p.a_src, p.a_dim, gr, k0 + it);
  } else {
    const int k = k0 + (lane & 15);
#pragma unroll
    for (int it = 0; it < 16; ++it) v[it] = a_value<AK>(p.a_src, p.a_dim, g_first + tw * 32 + it * 2 + (lane >> 4), k);
  }
}

template <AKind AK, bool SPLIT3>
__device__ __forceinline__ void a_store(const float (&v)[16], uint8_t* ah, uint8_t* al, int g_first, int k0, int tw,
                                        int lane) {
  const bool rows = a_rows_mapping<AK>(g_first, k0);
#pragma unroll
  for (int it = 0; it < 16; ++it) {
    const int r = rows ? tw * 32 + lane : tw * 32 + it * 2 + (lane >> 4);
    const int kl = rows ? it : (lane & 15);
    const uint32_t off = swz_offset(r, kl >> 2, 64) + (kl & 3) * 4;
    const float hi = tf32_hi(v[it]);
    *reinterpret_cast<float*>(ah + off) = hi;
    if constexpr (SPLIT3) *reinterpret_cast<float*>(al + off) = v[it] - hi;
  }
}

// Value of the structured right operand at (row k, column n); zero outside
// the n x n matrix.
template <BKind BK>
__device__ __forceinline__ float b_value(const float* __restrict__ src, int nd, int k, int n) {
  if (k >= nd || n >= nd) return 0.0f;
  if constexpr (BK == BKind::UpperPacked) {
    return n >= k ? __ldg(src + packed_idx(k, n, nd)) : 0.0f;
  } else {  // SymmPacked
    return n >= k ? __ldg(src + packed_idx(k, n, nd)) : __ldg(src + packed_idx(n, k, nd));
  }
}

// Byte offset of element (k-row kr, column n) in a B stage tile: 32-column
// boxes of 16 rows x 128 B, 128-byte swizzle with 32-byte atoms
// (32-byte granule index ^= row & 3).
__device__ __forceinline__ uint32_t b_tile_offset(uint32_t kr, uint32_t n) {
  const uint32_t j = n & 31u;
  return (n >> 5) * 2048u + kr * 128u + ((((j >> 3) ^ (kr & 3u))) << 5) + (j & 7u) * 4u;
}

template <AKind AK, BKind BK, bool SPLIT3, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const UmmaParams p) {
  constexpr int kBTile = TileGeom<BN>::kBTileBytes;
  constexpr int kStage = stage_bytes<BN, SPLIT3>();
  constexpr bool kATma = (AK == AKind::Dense || AK == AKind::UpperDense);
  constexpr bool kBTma = (BK == BKind::Dense);
  constexpr uint32_t kTxBytes = (kATma ? kATileBytes : 0) + (kBTma ? kBTile : 0);
  constexpr uint32_t kTmemCols = tmem_cols<BN, SPLIT3>();
  static_assert(!SPLIT3 || 3 * BN <= 512, "3xTF32 needs three BN-column regions of tensor memory");
  // A chunk's accumulator is folded when the transform warps reach stage
  // (c+1)*kChunk + kFoldLag: by then the MMAs of chunk c have completed
  // (the producer only refills a stage after its MMAs finish), and the fold
  // still precedes the first stage of chunk c+2, which reuses the buffer.
  constexpr int kFoldLag = STAGES - 1;
  static_assert(!SPLIT3 || kFoldLag <= kChunk, "fold lag must not exceed the chunk length");
  constexpr uint32_t kIdesc = make_idesc(kFmtTF32, kBM, BN, /*a_mn=*/0, /*b_mn=*/1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStage);
  uint64_t* ready = full + STAGES;
  uint64_t* empty = ready + STAGES;
  uint64_t* accum_full = empty + STAGES;
  uint64_t* acc_full = accum_full + 1;  // [2]: chunk finished in ping-pong buffer b
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto a_hi = [&](int s) { return smem + s * kStage; };
  auto b_hi = [&](int s) { return smem + s * kStage + kATileBytes; };
  auto a_lo = [&](int s) { return smem + s * kStage + kATileBytes + kBTile; };
  auto b_lo = [&](int s) { return smem + s * kStage + 2 * kATileBytes + kBTile; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Tile coordinates.  blockIdx.y walks row tiles first-to-last, so for the
  // triangular operand (whose row tile i has K range [128 i, N)) the longest
  // tiles are dispatched first.
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;
  const int m0 = m_tile * kBM;
  const int n0 = n_tile * BN;
  // Rows of a triangular operand are zero left of the diagonal: row tile
  // [g0, g0+128) of U needs k >= g0 only.
  int kb_begin = 0;
  if constexpr (AK == AKind::UpperPacked || AK == AKind::UpperDense) kb_begin = (p.a_row0 + m0) / kBK;
  int kb_end = (p.K + kBK - 1) / kBK;
  // An upper-triangular right operand is zero below its diagonal: column
  // tile [n0, n0+BN) needs k < n0 + BN only.
  if constexpr (BK == BKind::UpperPacked) kb_end = min(kb_end, (n0 + BN - 1) / kBK + 1);
  const int num_kb = kb_end - kb_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    if constexpr (kATma) tma_prefetch_desc(&tmA);
    if constexpr (kBTma) tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const bool tr = p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0;
  if (tr && threadIdx.x == 0) {
    p.trace[kTrTmem] = tmem_base;
    p.trace[kTrNumKb] = static_cast<uint32_t>(num_kb);
  }

  const WaitCtx wprod{abort_flag, p.status, p.wait_limit_ns, kWaitProducer};
  const WaitCtx wmma{abort_flag, p.status, p.wait_limit_ns, kWaitMma};
  const WaitCtx wxf{abort_flag, p.status, p.wait_limit_ns, kWaitTransform};
  const WaitCtx wepi{abort_flag, p.status, p.wait_limit_ns, kWaitEpilogue};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, wprod)) break;
        mbar_arrive_expect_tx(&full[s], kTxBytes);
        const int k0 = (kb_begin + i) * kBK;
        if constexpr (kATma) tma_load_2d(a_hi(s), &tmA, &full[s], k0, m0);
        if constexpr (kBTma) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
            tma_load_2d(b_hi(s) + c * TileGeom<BN>::kBChunkBytes, &tmB, &full[s], n0 + 32 * c, k0);
        }
        ++issued;
      }
      if (*abort_flag) {
        // Drain: wait (bounded, ignoring the abort flag) for the last copy
        // issued into each stage, so no bulk copy lands in shared memory
        // after the CTA has exited.
        volatile int no_abort = 0;
        const WaitCtx drain{&no_abort, p.status, p.wait_limit_ns, kWaitDrain};
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
          mbar_wait(&full[i % STAGES], (i / STAGES) & 1, drain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&ready[s], ph, wmma)) break;
        tc_fence_after_sync();
        const uint32_t sa = smem_u32(a_hi(s));
        const uint32_t sb = smem_u32(b_hi(s));
        // 3xTF32: chunk c = i / kChunk accumulates into buffer c & 1 and
        // starts from zero; otherwise one accumulator for the whole K.
        const bool chunk_start = SPLIT3 ? (i % kChunk == 0) : (i == 0);
        const uint32_t d_tmem = SPLIT3 ? tmem_base + static_cast<uint32_t>(((i / kChunk) & 1) * BN) : tmem_base;
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          // A: K-major, 64-byte rows, 8-row groups 512 B apart; a k-step of
          // 8 tf32 is 32 bytes along the row.
          const uint64_t da = make_smem_desc(sa + kk * 32, 16, 512, kLayoutSw64);
          // B: MN-major, 32-column boxes 2048 B apart (LBO), k-rows 128 B
          // apart in 4-row swizzle atoms 512 B apart (SBO); a k-step of 8
          // rows is 1024 B.
          const uint64_t db = make_smem_desc(sb + kk * 1024, TileGeom<BN>::kBChunkBytes, 512, kLayoutSw128Base32);
          const uint32_t acc = (!chunk_start || kk > 0) ? 1u : 0u;
          umma_tf32(d_tmem, da, db, kIdesc, acc);
          if constexpr (SPLIT3) {
            const uint32_t sal = smem_u32(a_lo(s));
            const uint32_t sbl = smem_u32(b_lo(s));
            const uint64_t dal = make_smem_desc(sal + kk * 32, 16, 512, kLayoutSw64);
            const uint64_t dbl =
                make_smem_desc(sbl + kk * 1024, TileGeom<BN>::kBChunkBytes, 512, kLayoutSw128Base32);
            umma_tf32(d_tmem, da, dbl, kIdesc, 1u);
            umma_tf32(d_tmem, dal, db, kIdesc, 1u);
          }
        }
        umma_commit(&empty[s]);
        if constexpr (SPLIT3) {
          if (i % kChunk == kChunk - 1 || i == num_kb - 1) umma_commit(&acc_full[(i / kChunk) & 1]);
        }
        if (tr && i == 0) {
          const uint64_t da = make_smem_desc(sa, 16, 512, kLayoutSw64);
          const uint64_t db = make_smem_desc(sb, TileGeom<BN>::kBChunkBytes, 512, kLayoutSw128Base32);
          p.trace[kTrDescA] = static_cast<uint32_t>(da);
          p.trace[kTrDescA + 1] = static_cast<uint32_t>(da >> 32);
          p.trace[kTrDescB] = static_cast<uint32_t>(db);
          p.trace[kTrDescB + 1] = static_cast<uint32_t>(db >> 32);
          p.trace[kTrIdesc] = kIdesc;
        }
        if (tr) p.trace[kTrMmas] = static_cast<uint32_t>(i + 1);
      }
      // Signals the epilogue; on abort it still fires once every MMA issued
      // so far has finished.  The issuer waits for it too (bounded, ignoring
      // the abort flag) so tensor memory is quiescent before it is freed.
      umma_commit(accum_full);
      volatile int no_abort = 0;
      const WaitCtx drain{&no_abort, p.status, p.wait_limit_ns, kWaitDrain};
      mbar_wait(accum_full, 0, drain);
    }
  } else {
    // ------------------------------------------------------------ transform
    const int t = threadIdx.x - 64;  // 0..127
    const int tw = t >> 5;           // transform warp 0..3
    bool ok = true;
    int folded = 0;                     // chunks already summed into the running sum
    const int g_first = p.a_row0 + m0;  // structured-A row of tile row 0
    float a_cur[16], a_nxt[16];
    if constexpr (!kATma) {
      if (num_kb > 0) a_gather<AK>(a_cur, p, g_first, kb_begin * kBK, tw, lane);
    }
    for (int i = 0; i < num_kb && ok; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      // Issue the next stage's global loads before waiting on this one: they
      // need no shared memory, so their latency overlaps the wait and the
      // stores below.
      if constexpr (!kATma) {
        if (i + 1 < num_kb) a_gather<AK>(a_nxt, p, g_first, (kb_begin + i + 1) * kBK, tw, lane);
      }
      if constexpr (SPLIT3) {
        if (i >= kChunk + kFoldLag && (i - kFoldLag) % kChunk == 0) {
          const int f = (i - kFoldLag) / kChunk - 1;  // chunk to fold
          if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[f & 1], (f >> 1) & 1, wxf))) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t lanes = static_cast<uint32_t>((warp & 3) * 32) << 16;
          const uint32_t src = tmem_base + lanes + static_cast<uint32_t>((f & 1) * BN);
          const uint32_t sum = tmem_base + lanes + static_cast<uint32_t>(2 * BN);
#pragma unroll 1
          for (int c = 0; c < BN; c += 16) {
            uint32_t r[16], q[16];
            tmem_ld_32x32b_x16(src + c, r);
            if (f > 0) tmem_ld_32x32b_x16(sum + c, q);
            tmem_wait_ld();
            if (f > 0) {
#pragma unroll
              for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
            }
            tmem_st_32x32b_x16(sum + c, r);
          }
          tmem_wait_st();
          tc_fence_before_sync();
          folded = f + 1;
        }
      }
      // Warp-uniform outcome: the tcgen05.ld below is .sync.aligned, so the
      // lanes of a warp must never take different paths.
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, wxf))) {
        ok = false;
        break;
      }
      const int k0 = (kb_begin + i) * kBK;
      if constexpr (!kATma) {
        a_store<AK, SPLIT3>(a_cur, a_hi(s), a_lo(s), g_first, k0, tw, lane);
#pragma unroll
        for (int j = 0; j < 16; ++j) a_cur[j] = a_nxt[j];
      } else if constexpr (SPLIT3) {
        const float4* src = reinterpret_cast<const float4*>(a_hi(s));
        float4* dst = reinterpret_cast<float4*>(a_lo(s));
#pragma unroll
        for (int j = t; j < kATileBytes / 16; j += 128) {
          const float4 x = src[j];
          dst[j] = make_float4(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y), x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
        }
      }
      if constexpr (!kBTma) {
        // Build the structured B tile: warp tw fills k-rows tw, tw+4, ...;
        // each lane one column of a 32-column box (coalesced along packed rows).
        uint8_t* bh = b_hi(s);
        uint8_t* bl = b_lo(s);
        // Symmetric tiles wholly below the diagonal (every column n < k) read
        // the mirror S[n][k]: 16 lanes along k per column keep those loads
        // coalesced along packed row n.
        const bool mirror = (BK == BKind::SymmPacked) && (n0 + BN <= k0);
        constexpr int kPer = (kBK * BN) / 128;  // elements per thread per stage
        constexpr int kBatch = kPer < 16 ? kPer : 16;
#pragma unroll 1
        for (int b0 = 0; b0 < kPer; b0 += kBatch) {
          float v[kBatch];
#pragma unroll
          for (int e = 0; e < kBatch; ++e) {
            const int q = b0 + e;  // 0 .. kPer-1
            int kr, n;
            if (mirror) {
              kr = lane & 15;
              n = (q * 4 + tw) * 2 + (lane >> 4);
            } else {
              kr = tw + 4 * (q / (BN / 32));
              n = (q % (BN / 32)) * 32 + lane;
            }
            v[e] = b_value<BK>(p.b_src, p.b_dim, k0 + kr, n0 + n);
          }
#pragma unroll
          for (int e = 0; e < kBatch; ++e) {
            const int q = b0 + e;
            int kr, n;
            if (mirror) {
              kr = lane & 15;
              n = (q * 4 + tw) * 2 + (lane >> 4);
            } else {
              kr = tw + 4 * (q / (BN / 32));
              n = (q % (BN / 32)) * 32 + lane;
            }
            const uint32_t off = b_tile_offset(kr, n);
            const float hi = tf32_hi(v[e]);
            *reinterpret_cast<float*>(bh + off) = hi;
            if constexpr (SPLIT3) *reinterpret_cast<float*>(bl + off) = v[e] - hi;
          }
        }
      } else if constexpr (SPLIT3) {
        const float4* src = reinterpret_cast<const float4*>(b_hi(s));
        float4* dst = reinterpret_cast<float4*>(b_lo(s));
#pragma unroll
        for (int j = t; j < kBTile / 16; j += 128) {
          const float4 x = src[j];
          dst[j] = make_float4(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y), x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
        }
      }
      if (tr && i == 0 && t == 0) {
        for (int j = 0; j < 8; ++j) {
          p.trace[kTrA + j] = reinterpret_cast<const uint32_t*>(a_hi(s))[j];
          p.trace[kTrB + j] = reinterpret_cast<const uint32_t*>(b_hi(s))[j];
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&ready[s]);
    }

    // ------------------------------------------------------------ epilogue
    const bool acc_ok = __all_sync(0xffffffffu, ok && mbar_wait(accum_full, 0, wepi) && !*abort_flag);
    if (tr && t == 0) p.trace[kTrAccOk] = acc_ok ? 1u : 0u;
    if (acc_ok) {
      tc_fence_after_sync();
      const int q = warp & 3;  // TMEM lanes 32q..32q+31 belong to this warp
      const int row = m0 + q * 32 + lane;
      const bool vec = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
      float* crow = p.C + static_cast<long long>(row) * p.ldc;
      const int nch = (num_kb + kChunk - 1) / kChunk;
      const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        if constexpr (SPLIT3) {
          // result = running sum (chunks [0, folded)) + the unfolded chunks
          // (at most two, in distinct ping-pong buffers).
          float acc[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
          if (folded > 0) {
            tmem_ld_32x32b_x16(tmem_base + lanes + 2 * BN + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = __uint_as_float(r[j]);
          }
#pragma unroll 1
          for (int f = folded; f < nch; ++f) {
            tmem_ld_32x32b_x16(tmem_base + lanes + static_cast<uint32_t>((f & 1) * BN) + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] += __uint_as_float(r[j]);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(acc[j]);
        } else {
          tmem_ld_32x32b_x16(tmem_base + lanes + c, r);
          tmem_wait_ld();
        }
        if (tr && q == 0 && lane == 0 && c == 0)
          for (int j = 0; j < 16; ++j) p.trace[kTrAcc + j] = r[j];
        const int col = n0 + c;
        if (row < p.M) {
          if (vec && col + 16 <= p.N) {
            float4* dst = reinterpret_cast<float4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          } else {
#pragma unroll
            for (int v = 0; v < 16; ++v)
              if (col + v < p.N) crow[col + v] = __uint_as_float(r[v]);
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace smm
