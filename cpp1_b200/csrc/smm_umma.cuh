// The tcgen05 contraction engine shared by every tensor-core operation of the
// library: C(M x N) = Aop(M x K) * B(K x N), fp32 row-major C, accumulator in
// tensor memory (TMEM).
//
// Tile: 128 x BN output per CTA (BN = 64, 128 or 256), K-blocks of 16 fp32
// (64 bytes) per pipeline stage, STAGES stages in shared memory.
//
// Operand staging per stage (hi = the fp32 value; kind::tf32 reads its upper
// 19 bits, i.e. truncates; lo = x - tf32(x), exact in fp32, computed in shared
// memory by the transform warps from the TMA-loaded tile, so only the raw
// operands cross L2):
//   A (K-major, 128 rows x 64 B, 64-byte swizzle):
//     AKind::Dense / UpperDense   TMA tile loads of a row-major A
//     AKind::UpperPacked          built on chip from packed-upper storage;
//                                 k-blocks left of the row tile's diagonal are
//                                 never visited
//     AKind::Toeplitz             built on chip from the 2N-1 generator (row r
//                                 of the tile is a contiguous window)
//     AKind::SymmPacked           built on chip from packed-upper storage,
//                                 mirrored below the diagonal
//     AKind::LowerPacked          built on chip from packed-lower storage
//                                 (idx(i,j) = i(i+1)/2 + j); k-blocks right of
//                                 the row tile's last diagonal element are
//                                 never visited
//   B (MN-major, BN columns x 16 k-rows, 32-column boxes, 128-byte swizzle
//     with 32-byte atoms — the only swizzle kind::tf32 accepts for an MN-major
//     operand; with the plain 128-byte swizzle the MMA produces nothing):
//     BKind::Dense                TMA tile loads of a row-major B
//     BKind::UpperPacked/SymmPacked/LowerPacked  built on chip (the DSL's
//                                 Gen@Upper, Gen@Symm, Symm@Symm, Gen@Lower,
//                                 Lower@Lower)
//     BKind::Toeplitz             built on chip from a K + N - 1 generator
//                                 (Gen@Toeplitz without room for a dense copy)
//
// 3xTF32 (SPLIT3): three MMAs per k-step, hi*hi + hi*lo + lo*hi.  The tensor
// core's fp32 accumulation truncates on every update, so with same-sign data
// its error grows with the number of updates into one accumulator.  The MMA
// therefore accumulates chunks of kChunk k-blocks, each starting from zero;
// at every chunk boundary the epilogue warps copy the accumulator to
// registers (the MMA waits only for that copy), then add it into a running
// sum kept in a second TMEM region with round-to-nearest fp32 adds while the
// next chunk runs.  Error stays ~1e-6 normwise whatever K is.
//
// Warp roles (384 threads):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2-9   transform (lo tiles, structured operand tiles), chunk folds, epilogue
//               (TMEM -> registers -> global C); warp w owns TMEM lanes
//               32*(w%4).. and column half (w-2)/4 of the tile
//   warps 10-11 structured-A fill (fp32 modes): 4-byte cp.async copies from
//               packed / generator storage straight into the swizzled A tile,
//               zero-filled outside the structure, completing on the stage's
//               `full` barrier (so the transform warps only derive lo tiles)
//
// Every wait is bounded (WaitCtx): on expiry the kernel records which role
// gave up in the status word, the other roles stop waiting, in-flight
// copies/MMAs are drained (bounded), TMEM is freed and the CTA exits.
#pragma once
#include <cuda_bf16.h>

#include "smm_device.cuh"

namespace smm {

enum class AKind : int { Dense = 0, UpperPacked = 1, Toeplitz = 2, SymmPacked = 3, UpperDense = 4, LowerPacked = 5 };
// Right operand: a dense row-major matrix loaded by TMA, or a packed
// upper-triangular / symmetric matrix built on chip by the transform warps.
enum class BKind : int { Dense = 0, UpperPacked = 1, SymmPacked = 2, LowerPacked = 3, Toeplitz = 4 };

// Arithmetic of the contraction (values match smm_mode).
enum class Mode : int { TF32x3 = 0, TF32 = 1, BF16 = 2 };

// Per-mode geometry.  A stage holds 64 bytes of K per A row in every mode
// (16 fp32 or 32 bf16) and a BN x 64-byte B tile:
//   fp32: B boxes of 32 columns x 16 k-rows (2 KiB), 128-byte swizzle with
//         32-byte atoms (descriptor layout 1), a k-step of 8 rows = 1 KiB;
//   bf16: B boxes of 64 columns x 32 k-rows (4 KiB), plain 128-byte swizzle
//         (layout 2), a k-step of 16 rows = 2 KiB.
template <Mode MD>
struct ModeTraits {
  static constexpr bool kSplit3 = (MD == Mode::TF32x3);
  static constexpr bool kBf16 = (MD == Mode::BF16);
  static constexpr int kElem = kBf16 ? 2 : 4;
  static constexpr int kStageK = 64 / kElem;        // K elements per stage
  static constexpr int kBoxCols = 128 / kElem;      // B box width (elements)
  static constexpr int kBoxRows = kStageK;          // B box height (k-rows)
  static constexpr int kBoxBytes = kBoxRows * 128;  // 2 or 4 KiB
  static constexpr uint32_t kBLayout = kBf16 ? kLayoutSw128 : kLayoutSw128Base32;
  static constexpr uint32_t kBSbo = kBf16 ? 1024 : 512;     // swizzle-atom row-group stride
  static constexpr uint32_t kBStepBytes = kBf16 ? 2048 : 1024;  // B bytes per MMA k-step
  static constexpr uint32_t kFmt = kBf16 ? kFmtBF16 : kFmtTF32;
};

// Structured A in fp32 modes is filled by cp.async warps (raw fp32, like a
// TMA tile).  In bf16 mode a Toeplitz block is staged the same way (the one
// generator window its 128 rows slide over, fp32) and converted by the
// transform warps; the other structured kinds are gathered and converted by
// the transform warps.
__host__ __device__ constexpr bool a_async_filled(AKind ak, Mode md) {
  return ak != AKind::Dense && ak != AKind::UpperDense && (md != Mode::BF16 || ak == AKind::Toeplitz);
}
__host__ __device__ constexpr bool a_staged(AKind ak, Mode md) { return ak == AKind::Toeplitz && md == Mode::BF16; }
// bf16 Toeplitz staging: the generator elements [lo, lo + 127 + 32 subs)
// that the 128 rows of `subs` consecutive k-blocks slide over (lo = n - 1 -
// (last row) + k0), from the 16-byte boundary at or below lo: 41 chunks of 16
// bytes for one k-block, 49 for two; a 1 KiB slot per k-block of the stage
// (stages stay 1 KiB aligned).
__host__ __device__ constexpr int stg_gen_chunks(int subs) { return (130 + 32 * subs + 3) / 4; }
constexpr int kStgBytes = 1024;
// Threads per CTA: producer, MMA and 8 transform warps, plus the 2 fill warps
// when the kernel has them.
__host__ __device__ constexpr int umma_threads(AKind ak, Mode md) { return a_async_filled(ak, md) ? 384 : 320; }

constexpr int kMaxMappedTiles = 64;  // row tiles of a mapped upper-triangular A (UmmaParams::a_tile_row0)

struct UmmaParams {
  int M, N, K;             // C is M x N; reduction length K
  float* C;                // row-major, leading dimension ldc
  int ldc;
  float* C_lo;             // optional: also store lo(C) = C - tf32(C) here (same ldc), so
                           // a following 3xTF32 product can read C as a split operand
  __nv_bfloat16* C_bf16;   // optional: also store bf16(C) here (leading dimension ldc_bf16),
  int ldc_bf16;            // so a following bf16 product can read C as an operand
  const float* a_src;      // packed U / generator / packed S (structured A kinds)
  int a_dim;               // order of the structured matrix
  int a_row0;              // row of the structured matrix that output row 0 maps to
  int a_lower;             // dense A is lower triangular: rows up to g need k <= g only
  int b_tri;               // dense B is upper (1) / lower (2) triangular: K range clipped per column tile
  const float* b_src;      // packed U / packed S (structured B kinds)
  int b_dim;               // order of the structured right operand
  int row_tiles;           // ceil(M / 128)
  int col_tiles;           // ceil(N / BN)
  int raster_group;        // row tiles per rasterisation group (L2 reuse)
  uint32_t* status;        // device status word (sticky error bits)
  unsigned long long wait_limit_ns;   // pipeline waits
  unsigned long long drain_limit_ns;  // teardown waits for copies / MMAs already issued (>= wait_limit_ns)
  uint32_t* trace;         // optional diagnostic record of CTA 0; null in normal use
  // Row-tile map of a dense-with-zeros upper-triangular A whose rows are a
  // stack of a_tile_rows-row tiles of U taken from anywhere in U: output row
  // tile i (of a_tile_rows rows) holds U's rows from a_tile_row0[i] on, so
  // its K range starts there.  a_tile_rows = 0: the rows are contiguous from
  // a_row0.
  int a_tile_rows;
  int a_tile_row0[kMaxMappedTiles];
};

// U's row behind output row r0 (a row-tile map, or contiguous from a_row0).
__device__ __forceinline__ int a_struct_row(const UmmaParams& p, int r0) {
  if (p.a_tile_rows > 0) return p.a_tile_row0[r0 / p.a_tile_rows] + r0 % p.a_tile_rows;
  return p.a_row0 + r0;
}

// Slots of the diagnostic record (UmmaParams::trace, 64 words).
enum : int {
  kTrTmem = 0,
  kTrNumKb = 1,
  kTrAccOk = 2,
  kTrMmas = 3,
  kTrAcc = 4 /*16 words*/,
  kTrTime = 24 /*8 phase stamps (low 32 bits of %globaltimer, ns) of CTA 0, then 8 of the grid's last CTA*/,
  kTrWords = 64
};

constexpr int kBM = 128;
constexpr int kBK = 16;                     // fp32 elements per k-block (64 bytes)
constexpr int kXformThreads = 256;          // warps 2-9
constexpr int kAFillThreads = 64;           // warps 10-11 (structured A, fp32 modes)
constexpr int kATileBytes = kBM * kBK * 4;  // 8 KiB
// 3xTF32 chunk length in k-blocks: 3 * 12 * 2 = 72 truncating updates per
// chunk accumulator (measured bias ~5e-8 of |C| per update on same-sign data).
constexpr int kChunk = 12;

template <int BN>
struct TileGeom {
  static constexpr int kBTileBytes = BN * kBK * 4;  // BN/32 boxes of 16 rows x 128 B
  static constexpr int kBChunkBytes = 16 * 128;     // one 32-column box
};

template <int BN, bool SPLIT3, bool STAGING = false>
__host__ __device__ constexpr int stage_bytes() {
  return (SPLIT3 ? 2 : 1) * (kATileBytes + TileGeom<BN>::kBTileBytes) + (STAGING ? kStgBytes : 0);
}

template <int BN, bool SPLIT3>
__host__ __device__ constexpr uint32_t tmem_cols() {
  // SPLIT3: chunk accumulator [0,BN) and running sum [BN,2BN)
  return SPLIT3 ? (2 * BN <= 128 ? 128u : (2 * BN <= 256 ? 256u : 512u)) : (BN < 32 ? 32u : static_cast<uint32_t>(BN));
}

// k-blocks (64 bytes of K each) per pipeline stage.  Two wherever the
// two-block stage still fits three times into 192 KiB (four for the one-pass
// modes on TMA-fed operands): every barrier round trip, wait and commit of
// the serial MMA-issuing thread then covers 4 (8) MMAs per pass instead of 2.
// Each of those instructions costs that thread ~60 cycles, about half of a
// 2-MMA stage's tensor time in one-pass modes.  3xTF32 with three blocks (two
// stages) measured slower.  bf16 structured A, gathered through registers one
// k-block at a time, keeps one; bf16 Toeplitz A, staged as one generator
// window per stage, takes two (the MMA issuer's overhead per stage is then
// spread over 4 MMAs, and the window grows by 32 elements only).
template <AKind AK, Mode MD, int BCOLS>
__host__ __device__ constexpr int umma_subs() {
  return (AK == AKind::Toeplitz && MD == Mode::BF16)
             ? 2
         : (AK != AKind::Dense && AK != AKind::UpperDense && MD == Mode::BF16)
             ? 1
             : ((AK == AKind::Dense || AK == AKind::UpperDense) && MD != Mode::TF32x3 &&
                3 * 4 * stage_bytes<BCOLS, false>() <= 192 * 1024)
                   ? 4  // one-pass modes on TMA-fed operands: 8 MMAs per stage
                   : (3 * 2 * stage_bytes<BCOLS, MD == Mode::TF32x3>() <= 192 * 1024 ? 2 : 1);
}
// Bytes of one pipeline stage.
template <AKind AK, Mode MD, int BCOLS>
__host__ __device__ constexpr int umma_stage_bytes() {
  return umma_subs<AK, MD, BCOLS>() * stage_bytes<BCOLS, MD == Mode::TF32x3, a_staged(AK, MD)>();
}
// Pipeline stages: as many as fit into 192 KiB, at most 8.
template <AKind AK, Mode MD, int BCOLS>
__host__ __device__ constexpr int umma_stages() {
  return (192 * 1024 / umma_stage_bytes<AK, MD, BCOLS>()) > 8 ? 8 : 192 * 1024 / umma_stage_bytes<AK, MD, BCOLS>();
}
template <AKind AK, Mode MD, int BCOLS, int STAGES>
__host__ __device__ constexpr int umma_smem_bytes() {
  return 1024 /*alignment slack*/ + STAGES * umma_stage_bytes<AK, MD, BCOLS>() + 256 /*barriers etc*/;
}

__device__ __forceinline__ long long packed_idx(long long i, long long j, long long n) {
  return i * n - i * (i - 1) / 2 + (j - i);
}

// Elements of a packed triangle of order n.
__device__ __forceinline__ long long packed_len(long long n) { return n * (n + 1) / 2; }

// Value of the structured right operand at (row k, column n); zero outside.
template <BKind BK>
__device__ __forceinline__ float b_value(const float* __restrict__ src, int nd, int k, int n, uint32_t* status) {
  if (k >= nd || n >= nd) return 0.0f;
  const long long len = packed_len(nd);
  if constexpr (BK == BKind::UpperPacked) {
    return n >= k ? ld_chk(src, packed_idx(k, n, nd), len, status, kBoundsB) : 0.0f;
  } else if constexpr (BK == BKind::LowerPacked) {
    return n <= k ? ld_chk(src, static_cast<long long>(k) * (k + 1) / 2 + n, len, status, kBoundsB) : 0.0f;
  } else {  // SymmPacked
    return ld_chk(src, n >= k ? packed_idx(k, n, nd) : packed_idx(n, k, nd), len, status, kBoundsB);
  }
}

// Byte offset of element (k-row kr, column n) in a B stage tile: 32-column
// boxes of 16 rows x 128 B, 128-byte swizzle with 32-byte atoms (32-byte
// granule index ^= row & 3).
__device__ __forceinline__ uint32_t b_tile_offset(uint32_t kr, uint32_t n) {
  const uint32_t j = n & 31u;
  return (n >> 5) * 2048u + kr * 128u + ((((j >> 3) ^ (kr & 3u))) << 5) + (j & 7u) * 4u;
}

// ---------------------------------------------------------------- structured A
// The 8 values one transform thread contributes to a structured A stage tile
// (rows m0.., columns k0..k0+15), gathered into registers so all loads are in
// flight together (latency, not bandwidth, bounds this producer).
//   lanes along k (16 lanes per row, two rows per warp instruction): rows
//     xw*16 + 2*it + lane/16, column lane%16 — coalesced along a packed row
//     or a generator window;
//   lanes along rows (symmetric tiles wholly below the diagonal, whose
//     elements are the mirror S[k][row]): row (xw%4)*32 + lane, column
//     (xw/4)*8 + it — coalesced along packed row k.
template <AKind AK, int KS>
__device__ __forceinline__ bool a_rows_mapping(int g_first, int k0) {
  return AK == AKind::SymmPacked && k0 + KS <= g_first;
}

// KS = K elements per stage (16 fp32 or 32 bf16): 128*KS/256 = KS/2
// elements per thread; KS/16 k-columns per lane group in the k mapping.
template <int KS>
__device__ __forceinline__ void a_coord(bool rows, int xw, int lane, int it, int& r, int& kl) {
  if (rows) {
    r = (xw & 3) * 32 + lane;
    kl = (xw >> 2) * (KS / 2) + it;
  } else if (KS == 16) {
    r = xw * 16 + it * 2 + (lane >> 4);
    kl = lane & 15;
  } else {  // 32: one row per warp instruction
    r = xw * 16 + it;
    kl = lane;
  }
}

// Offset of element (gr, 0) in the operand's storage for the rows a thread
// gathers in the k mapping (fixed for the whole K loop): packed upper
// row start minus gr, or n - 1 - gr for a Toeplitz generator, so the element
// (gr, k) is src[base + k].  Packed storage of order n < 92682 has fewer than
// 2^32 elements (the host rejects larger), so offsets are 32-bit; an
// out-of-range row's base may wrap but is never dereferenced.
__device__ __forceinline__ uint32_t packed_row_base(long long i, long long n) {
  return static_cast<uint32_t>(i * n - i * (i - 1) / 2 - i);
}
// Same for packed-lower storage: element (i, k), k <= i, at i(i+1)/2 + k.
__device__ __forceinline__ uint32_t lower_row_base(long long i) { return static_cast<uint32_t>(i * (i + 1) / 2); }

template <AKind AK, int KS>
__device__ __forceinline__ void a_row_bases(uint32_t (&rb)[KS / 2], const UmmaParams& p, int g_first, int xw,
                                            int lane) {
#pragma unroll
  for (int it = 0; it < KS / 2; ++it) {
    int r, kl;
    a_coord<KS>(false, xw, lane, it, r, kl);
    const long long gr = g_first + r;
    rb[it] = (AK == AKind::Toeplitz)      ? static_cast<uint32_t>(p.a_dim - 1 - gr)
             : (AK == AKind::LowerPacked) ? lower_row_base(gr)
                                          : packed_row_base(gr, p.a_dim);
  }
}

// Elements of a structured left operand of order n: a Toeplitz generator
// (2n - 1) or a packed triangle.
template <AKind AK>
__device__ __forceinline__ long long a_src_len(long long n) {
  return AK == AKind::Toeplitz ? 2 * n - 1 : packed_len(n);
}

template <AKind AK, int KS>
__device__ __forceinline__ void a_gather(float (&v)[KS / 2], const UmmaParams& p, const uint32_t (&rb)[KS / 2],
                                         int g_first, int k0, int xw, int lane) {
  const int n = p.a_dim;
  const float* __restrict__ src = p.a_src;
  const long long len = a_src_len<AK>(n);
  if (a_rows_mapping<AK, KS>(g_first, k0)) {
    // symmetric tile wholly below the diagonal: element (gr, k) = S[k][gr],
    // at row start of packed row k (+ gr), k consecutive per thread
    int r, kl;
    a_coord<KS>(true, xw, lane, 0, r, kl);
    const int gr = g_first + r;
    uint32_t base = packed_row_base(k0 + kl, n);
#pragma unroll
    for (int it = 0; it < KS / 2; ++it) {
      const int k = k0 + kl + it;
      v[it] = (gr < n && k < n) ? ld_chk(src, base + static_cast<uint32_t>(gr), len, p.status, kBoundsA) : 0.0f;
      base += static_cast<uint32_t>(n - k - 1);  // row start of packed row k+1
    }
    return;
  }
  int r0, kl;
  a_coord<KS>(false, xw, lane, 0, r0, kl);
  const int k = k0 + kl;
  uint32_t mbase = 0;  // symmetric, below-diagonal elements: packed row k
  if constexpr (AK == AKind::SymmPacked) mbase = packed_row_base(k, n);
#pragma unroll
  for (int it = 0; it < KS / 2; ++it) {
    int r;
    a_coord<KS>(false, xw, lane, it, r, kl);
    const int gr = g_first + r;
    const bool in = gr < n && k < n;
    if constexpr (AK == AKind::UpperPacked) {
      v[it] = (in && k >= gr) ? ld_chk(src, rb[it] + static_cast<uint32_t>(k), len, p.status, kBoundsA) : 0.0f;
    } else if constexpr (AK == AKind::LowerPacked) {
      v[it] = (in && k <= gr) ? ld_chk(src, rb[it] + static_cast<uint32_t>(k), len, p.status, kBoundsA) : 0.0f;
    } else if constexpr (AK == AKind::Toeplitz) {
      v[it] = in ? ld_chk(src, rb[it] + static_cast<uint32_t>(k), len, p.status, kBoundsA) : 0.0f;
    } else {
      v[it] = in ? ld_chk(src, k >= gr ? rb[it] + static_cast<uint32_t>(k) : mbase + static_cast<uint32_t>(gr), len,
                          p.status, kBoundsA)
                 : 0.0f;
    }
  }
}

template <AKind AK, Mode MD>
__device__ __forceinline__ void a_store(const float (&v)[ModeTraits<MD>::kStageK / 2], uint8_t* ah, uint8_t* al,
                                        int g_first, int k0, int xw, int lane) {
  using T = ModeTraits<MD>;
  constexpr int KS = T::kStageK;
  const bool rows = a_rows_mapping<AK, KS>(g_first, k0);
#pragma unroll
  for (int it = 0; it < KS / 2; ++it) {
    int r, kl;
    a_coord<KS>(rows, xw, lane, it, r, kl);
    if constexpr (T::kBf16) {
      const uint32_t off = swz_offset(r, kl >> 3, 64) + (kl & 7) * 2;
      *reinterpret_cast<__nv_bfloat16*>(ah + off) = __float2bfloat16_rn(v[it]);
    } else {
      const uint32_t off = swz_offset(r, kl >> 2, 64) + (kl & 3) * 4;
      const float hi = tf32_hi(v[it]);
      *reinterpret_cast<float*>(ah + off) = hi;
      if constexpr (T::kSplit3) *reinterpret_cast<float*>(al + off) = v[it] - hi;
    }
  }
}

// Fill this CTA's A stage tile (128 rows x 16 fp32, rows g_first.., columns
// k0..k0+15, 64-byte swizzle) from structured storage with 4-byte cp.async
// copies; fill thread `ft` of kAFillThreads issues 32.  Lanes run along k
// (16 lanes per row, two rows per warp instruction: coalesced along a packed
// row or a generator window), except for symmetric tiles wholly below the
// diagonal, whose elements are mirrors S[k][row]: there 32 lanes run along
// rows (coalesced along packed row k).  Elements outside the matrix or
// below an upper-triangular diagonal are written as zeros without a read.
template <AKind AK>
__device__ __forceinline__ void a_async_fill(const UmmaParams& p, uint8_t* ah, int g_first, int k0, int ft) {
  constexpr int KS = 16;
  const int n = p.a_dim;
  const float* __restrict__ src = p.a_src;
  const uint32_t dst0 = smem_u32(ah);
  const int fw = ft >> 5, lane = ft & 31;
  const long long len = a_src_len<AK>(n);
  if (a_rows_mapping<AK, KS>(g_first, k0)) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int kl = fw * 8 + kk;
      const int k = k0 + kl;
      const uint32_t kb = packed_row_base(k, n);  // S[k][gr] = src[kb + gr]
#pragma unroll
      for (int rg = 0; rg < 4; ++rg) {
        const int r = rg * 32 + lane;
        const int gr = g_first + r;
        const bool in = gr < n && k < n && dbg_ok(kb + static_cast<uint32_t>(gr), len, p.status, kBoundsA);
        cp_async_4(dst0 + swz_offset(r, kl >> 2, 64) + (kl & 3) * 4, in ? src + (kb + static_cast<uint32_t>(gr)) : src,
                   in ? 4u : 0u);
      }
    }
    return;
  }
  const int kl = lane & 15;
  const int k = k0 + kl;
  uint32_t mbase = 0;  // symmetric, below-diagonal elements: packed row k
  if constexpr (AK == AKind::SymmPacked) mbase = packed_row_base(k, n);
  int r = fw * 64 + (lane >> 4);
  int gr = g_first + r;
  // offset of element (gr, 0): packed row start minus gr, lower row start, or n - 1 - gr
  uint32_t rb = (AK == AKind::Toeplitz)      ? static_cast<uint32_t>(n - 1 - gr)
                : (AK == AKind::LowerPacked) ? lower_row_base(gr)
                                             : packed_row_base(gr, n);
#pragma unroll 8
  for (int it = 0; it < 32; ++it) {
    const bool in = gr < n && k < n;
    bool valid;
    uint32_t so;
    if constexpr (AK == AKind::UpperPacked) {
      valid = in && k >= gr;
      so = rb + static_cast<uint32_t>(k);
    } else if constexpr (AK == AKind::LowerPacked) {
      valid = in && k <= gr;
      so = rb + static_cast<uint32_t>(k);
    } else if constexpr (AK == AKind::Toeplitz) {
      valid = in;
      so = rb + static_cast<uint32_t>(k);
    } else {
      valid = in;
      so = k >= gr ? rb + static_cast<uint32_t>(k) : mbase + static_cast<uint32_t>(gr);
    }
    valid = valid && dbg_ok(so, len, p.status, kBoundsA);
    cp_async_4(dst0 + swz_offset(r, kl >> 2, 64) + (kl & 3) * 4, valid ? src + so : src, valid ? 4u : 0u);
    // next row of this lane: two rows down
    if constexpr (AK == AKind::Toeplitz)
      rb -= 2u;
    else if constexpr (AK == AKind::LowerPacked)
      rb += static_cast<uint32_t>(2 * gr + 3);  // lower row base(gr + 2) - base(gr)
    else
      rb += static_cast<uint32_t>(2 * n - 2 * gr - 3);  // packed row base(gr + 2) - base(gr)
    r += 2;
    gr += 2;
  }
}

// ---------------------------------------------------------------- Toeplitz A, bf16
// Generator index of element (g_first + 127, k0), the lowest one a k-block of
// the tile reads (negative when the window starts before the generator).
__device__ __forceinline__ long long toeplitz_lo(long long n, int g_first, int k0) {
  return n - 1 - (g_first + kBM - 1) + k0;
}

// Stage the generator window of SUBS bf16 k-blocks (32 SUBS k from k0) of
// this CTA's Toeplitz rows g_first..: stg_gen_chunks(SUBS) aligned 16-byte
// chunks, one per fill thread.  A chunk wholly outside the generator
// [g, g + 2n - 1) is skipped (the conversion never reads it); one that
// overlaps either end is copied element by element, so no byte outside the
// generator is read.
template <int SUBS>
__device__ __forceinline__ void a_stage_fill_toeplitz_bf16(const UmmaParams& p, uint8_t* stg, int g_first, int k0,
                                                           int ft) {
  static_assert(stg_gen_chunks(SUBS) <= kAFillThreads && 16 * stg_gen_chunks(SUBS) <= SUBS * kStgBytes,
                "window chunks: one per fill thread, inside the stage's slots");
  if (ft >= stg_gen_chunks(SUBS)) return;
  const long long n = p.a_dim;
  const uintptr_t b = reinterpret_cast<uintptr_t>(p.a_src);
  const uintptr_t e = b + 4 * static_cast<uintptr_t>(2 * n - 1);
  const uintptr_t a16 = ((b + 4 * toeplitz_lo(n, g_first, k0)) & ~uintptr_t(15)) + 16 * static_cast<uintptr_t>(ft);
  const uint32_t dst = smem_u32(stg) + 16 * ft;
  if (a16 + 16 <= b || a16 >= e) return;
  if (a16 >= b && a16 + 16 <= e) {
    cp_async_16(dst, reinterpret_cast<const void*>(a16));
    return;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uintptr_t x = a16 + 4 * j;
    if (x >= b && x < e) cp_async_4(dst + 4 * j, reinterpret_cast<const float*>(x), 4u);
  }
}

// bf16 A tile (128 rows x 32 k, 64-byte swizzle) of the k-block at
// k0 + jofs from the window staged for the stage starting at k0: element
// (row r, k0 + jofs + kk) is window element (127 - r) + jofs + kk.  Each
// transform thread converts 4 groups of 4 consecutive k of one row (rows
// t/8 + 32 it, columns 4 (t % 8)..), zero outside the matrix.
__device__ __forceinline__ void a_stage_convert_toeplitz_bf16(const UmmaParams& p, const uint8_t* stg, uint8_t* ah,
                                                              int g_first, int k0, int jofs, int t) {
  const long long n = p.a_dim;
  const float* sf = reinterpret_cast<const float*>(stg);
  const int off =
      static_cast<int>(((reinterpret_cast<uintptr_t>(p.a_src) + 4 * toeplitz_lo(n, g_first, k0)) & 15) >> 2);
  const int q = t & 7, kk0 = 4 * q;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 32 + (t >> 3);
    const bool row_in = g_first + r < n;
    const float* w = sf + off + (kBM - 1 - r) + jofs + kk0;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = (row_in && k0 + jofs + kk0 + j < n) ? w[j] : 0.0f;
    __nv_bfloat162 lo2 = __floats2bfloat162_rn(v[0], v[1]), hi2 = __floats2bfloat162_rn(v[2], v[3]);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo2);
    pk.y = *reinterpret_cast<uint32_t*>(&hi2);
    *reinterpret_cast<uint2*>(ah + swz_offset(r, kk0 >> 3, 64) + (kk0 & 7) * 2) = pk;
  }
}

// ---------------------------------------------------------------- structured B
// Element e (0 .. BN/16-1) of transform thread t in a B stage tile.  Lanes
// run along n (coalesced along packed row k); for symmetric tiles wholly
// below the diagonal (every n < k, elements are the mirror S[n][k]) 16 lanes
// run along k instead (coalesced along packed row n).
// KS = k-rows per stage (16 fp32, 32 bf16).
template <int BN, int KS>
__device__ __forceinline__ void b_coord(bool mirror, int t, int e, int& kr, int& n) {
  const int xw = t >> 5, lane = t & 31;
  if (mirror) {
    if (KS == 16) {
      kr = lane & 15;
      n = (e * 8 + xw) * 2 + (lane >> 4);
    } else {
      kr = lane;
      n = e * 8 + xw;
    }
  } else {
    const int lin = e * kXformThreads + t;
    kr = lin / BN;
    n = lin % BN;
  }
}

// Byte offset of (k-row kr, column n) in a bf16 B stage tile: 64-column boxes
// of 32 rows x 128 B, plain 128-byte swizzle (16-byte chunk index ^= row & 7).
__device__ __forceinline__ uint32_t b_tile_offset_bf16(uint32_t kr, uint32_t n) {
  const uint32_t j = n & 63u;
  return (n >> 6) * 4096u + kr * 128u + (((j >> 3) ^ (kr & 7u)) << 4) + (j & 7u) * 2u;
}

template <BKind BK, int BN, Mode MD>
__device__ __forceinline__ void b_build(const UmmaParams& p, uint8_t* bh, uint8_t* bl, int k0, int n0, int t) {
  using T = ModeTraits<MD>;
  constexpr int KS = T::kStageK;
  const bool mirror = (BK == BKind::SymmPacked) && (n0 + BN <= k0);
  constexpr int kPer = (KS * BN) / kXformThreads;
  constexpr int kBatch = kPer < 16 ? kPer : 16;
#pragma unroll 1
  for (int b0 = 0; b0 < kPer; b0 += kBatch) {
    float v[kBatch];
#pragma unroll
    for (int e = 0; e < kBatch; ++e) {
      int kr, n;
      b_coord<BN, KS>(mirror, t, b0 + e, kr, n);
      if constexpr (BK == BKind::Toeplitz) {  // K x N Toeplitz of generator b_src: T[k][n] = g[(K-1) + (n-k)]
        const int k = k0 + kr, nn = n0 + n;
        v[e] = (k < p.K && nn < p.N)
                   ? ld_chk(p.b_src, static_cast<long long>(p.K) - 1 + nn - k,
                            static_cast<long long>(p.K) + p.N - 1, p.status, kBoundsB)
                   : 0.0f;
      } else {
        v[e] = b_value<BK>(p.b_src, p.b_dim, k0 + kr, n0 + n, p.status);
      }
    }
#pragma unroll
    for (int e = 0; e < kBatch; ++e) {
      int kr, n;
      b_coord<BN, KS>(mirror, t, b0 + e, kr, n);
      if constexpr (T::kBf16) {
        *reinterpret_cast<__nv_bfloat16*>(bh + b_tile_offset_bf16(kr, n)) = __float2bfloat16_rn(v[e]);
      } else {
        const uint32_t off = b_tile_offset(kr, n);
        const float hi = tf32_hi(v[e]);
        *reinterpret_cast<float*>(bh + off) = hi;
        if constexpr (T::kSplit3) *reinterpret_cast<float*>(bl + off) = v[e] - hi;
      }
    }
  }
}

// ---------------------------------------------------------------- kernel
// tmA/tmB map the operands (hi, or bf16 copies), tmAl/tmBl their lo planes
// (3xTF32 only).
//
// PAIR: the CTA pair form.  Clusters of two CTAs compute a 256 x BN tile with
// tcgen05.mma.cta_group::2 issued by the even CTA (the leader): each CTA
// stages its own 128 A rows and BN/2 B columns (so per SM the MMA reads 1.5x
// fewer shared-memory bytes per flop than the one-CTA 128 x BN tile, and the
// stage is smaller, so more stages fit), and holds its 128 rows of the
// accumulator in its own tensor memory.  Each CTA's TMA completes on its own
// `full` barrier; its transform warps then arrive on the leader's `ready`
// barrier, the leader's MMA commits to the `empty`,
// `acc_full` and `accum_full` barriers of both CTAs (one commit per CTA), and
// the fold warps of both CTAs arrive on the leader's `acc_empty`.  No load is
// multicast.
//
// SPLITK (single-CTA tiles only): clusters of SPLITK = 2 CTAs compute the
// same 128 x BN tile over the two halves of its k-block range (whole stages
// each), each in its own tensor memory with its own pipeline.  After both
// pipelines are done, CTA 1 writes its result rows into CTA 0's stage memory
// (distributed shared memory), and CTA 0 adds them to its own, in that fixed
// order, and stores C: twice the CTAs for a product with few output tiles,
// the same result on every run.
template <AKind AK, BKind BK, Mode MD, int BN, int STAGES, bool PAIR = false, int SPLITK = 1>
__global__ void __launch_bounds__(umma_threads(AK, MD), 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmAl, const __grid_constant__ CUtensorMap tmBl,
                     const UmmaParams p) {
  static_assert(SPLITK == 1 || (SPLITK == 2 && !PAIR), "split-K clusters of two single-CTA tiles");
  using MT = ModeTraits<MD>;
  constexpr bool SPLIT3 = MT::kSplit3;
  constexpr int KS = MT::kStageK;
  constexpr int kBCols = PAIR ? BN / 2 : BN;  // B columns staged by this CTA
  constexpr int kBTile = TileGeom<kBCols>::kBTileBytes;
  // A stage holds kSubs k-blocks of KS: [A hi x kSubs | B hi x kSubs | A lo x
  // kSubs | B lo x kSubs], each block in the one-block layouts below.
  constexpr int kSubs = umma_subs<AK, MD, kBCols>();
  constexpr bool kStaging = a_staged(AK, MD);  // bf16 Toeplitz: fp32 generator window after the tiles
  static_assert(!kStaging || kSubs <= 2, "staged A: one generator window per stage");
  constexpr int kStage = umma_stage_bytes<AK, MD, kBCols>();
  constexpr int kChunkS = kChunk / kSubs;  // chunk length in stages
  static_assert(kChunk % kSubs == 0, "chunk of whole stages");
  constexpr bool kATma = (AK == AKind::Dense || AK == AKind::UpperDense);
  constexpr bool kBTma = (BK == BKind::Dense);
  constexpr bool kACp = a_async_filled(AK, MD);
  // The transform warps touch every stage when a tile is built on chip or
  // when lo tiles are derived from the loaded ones (3xTF32); in a pair they
  // also relay stage completion to the leader.
  constexpr bool kXform = !kATma || !kBTma || SPLIT3 || PAIR;
  constexpr uint32_t kTxBytes = kSubs * ((kATma ? kATileBytes : 0) + (kBTma ? kBTile : 0));
  constexpr uint32_t kTmemCols = tmem_cols<BN, SPLIT3>();
  constexpr uint32_t kIdesc = make_idesc(MT::kFmt, PAIR ? 2 * kBM : kBM, BN, /*a_mn=*/0, /*b_mn=*/1);
  constexpr int kHalf = BN / 2;  // columns per epilogue warp
  constexpr uint32_t kArrivals = (PAIR ? 2 : 1) * (kXformThreads / 32);  // warps arriving on ready / acc_empty
  constexpr int kFoldLag = STAGES / 2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStage);
  uint64_t* ready = full + STAGES;
  uint64_t* empty = ready + STAGES;
  uint64_t* accum_full = empty + STAGES;  // every MMA done
  uint64_t* acc_full = accum_full + 1;    // chunk c done (phase c)
  uint64_t* acc_empty = acc_full + 1;     // chunk c copied out of the accumulator (phase c)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  auto a_hi = [&](int s) { return smem + s * kStage; };
  auto b_hi = [&](int s) { return smem + s * kStage + kSubs * kATileBytes; };
  auto a_lo = [&](int s) { return smem + s * kStage + kSubs * (kATileBytes + kBTile); };
  auto b_lo = [&](int s) { return smem + s * kStage + kSubs * (2 * kATileBytes + kBTile); };
  auto stg = [&](int s) { return smem + s * kStage + kSubs * (kATileBytes + kBTile); };  // bf16 only

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const uint32_t krank = SPLITK > 1 ? cluster_ctarank() : 0u;  // this CTA's half of the K range
  const bool leader = (rank == 0);
  // shared::cluster address of a barrier of this CTA in CTA `r` of the pair
  auto in_cta = [&](uint64_t* bar, uint32_t r) { return mapa_shared(smem_u32(bar), r); };

  // Grouped rasterisation: consecutive tiles cover raster_group row tiles x
  // all column tiles, so a wave shares A and B slices through L2.  Groups go
  // top to bottom, so for the triangular operand (row tile i has K range
  // [tile height * i, N)) the longest tiles are dispatched first.  In a pair,
  // a row tile is 256 rows and both CTAs take the same tile.
  int m_tile, n_tile;
  {
    const int b = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x) / SPLITK;
    const int per_group = p.raster_group * p.col_tiles;
    const int g = b / per_group;
    const int first = g * p.raster_group;
    const int rows_here = min(p.raster_group, p.row_tiles - first);
    const int in = b - g * per_group;
    m_tile = first + in % rows_here;
    n_tile = in / rows_here;
  }
  const int tile_m0 = m_tile * (PAIR ? 2 * kBM : kBM);
  const int m0 = tile_m0 + static_cast<int>(rank) * kBM;   // this CTA's A rows / C rows
  const int n0 = n_tile * BN;                              // the tile's columns
  const int nb0 = n0 + static_cast<int>(rank) * kBCols;    // this CTA's B columns
  // Rows of a triangular left operand are zero left of the diagonal: a row
  // tile starting at row g0 needs k >= g0 only.
  int kb_begin = 0;
  if constexpr (AK == AKind::UpperPacked) kb_begin = (p.a_row0 + tile_m0) / KS;
  if constexpr (AK == AKind::UpperDense) kb_begin = a_struct_row(p, tile_m0) / KS;
  int kb_end = (p.K + KS - 1) / KS;
  // A lower-triangular left operand is zero right of its diagonal: rows up
  // to g1 need k <= g1 only.
  if (AK == AKind::LowerPacked || (AK == AKind::Dense && p.a_lower))
    kb_end = min(kb_end, (p.a_row0 + tile_m0 + (PAIR ? 2 * kBM : kBM) - 1) / KS + 1);
  // An upper-triangular right operand is zero below its diagonal: column
  // tile [n0, n0+BN) needs k < n0 + BN only; a lower-triangular one is zero
  // above it: the tile needs k >= n0 only.
  if (BK == BKind::UpperPacked || (BK == BKind::Dense && p.b_tri == 1)) kb_end = min(kb_end, (n0 + BN - 1) / KS + 1);
  if (BK == BKind::LowerPacked || (BK == BKind::Dense && p.b_tri == 2)) kb_begin = max(kb_begin, n0 / KS);
  if constexpr (SPLITK > 1) {
    // Runs of whole stages, so neither CTA reads into the other's k-blocks.
    const int total = max(kb_end - kb_begin, 0);
    const int per = ((total + SPLITK - 1) / SPLITK + kSubs - 1) / kSubs * kSubs;
    const int b0 = kb_begin + static_cast<int>(krank) * per;
    kb_end = min(kb_end, b0 + per);
    kb_begin = min(b0, kb_end);
  }
  // Empty for a tile of L1 L2 wholly above the diagonal: it is written as
  // zeros.  num_kb counts stages of kSubs k-blocks; a last stage reaching
  // past kb_end multiplies zeros (past K, past a triangle's diagonal).
  const int num_kb = (max(kb_end - kb_begin, 0) + kSubs - 1) / kSubs;
  const int nch = SPLIT3 ? (num_kb + kChunkS - 1) / kChunkS : 1;

  // Phase stamps of the diagnostic record (CTA 0 and the grid's last CTA).
  const int trb = p.trace == nullptr ? -1 : blockIdx.x == 0 ? 0 : blockIdx.x == gridDim.x - 1 ? 1 : -1;
  auto stamp = [&](int i) {
    if (trb >= 0) p.trace[kTrTime + 8 * trb + i] = static_cast<uint32_t>(globaltimer_ns());
  };
  if (threadIdx.x == 0) stamp(0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1 + (kACp ? kAFillThreads : 0));  // TMA producer (+ fill threads)
      mbar_init(&ready[s], kArrivals);  // one arrival per transform warp (of both CTAs)
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kArrivals);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    if constexpr (kATma) tma_prefetch_desc(&tmA);
    if constexpr (kBTma) tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_alloc_pair(tmem_slot, kTmemCols);
    else
      tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before_sync();
  if constexpr (PAIR)
    cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival
  else
    __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) stamp(1);
  const bool tr = p.trace != nullptr && blockIdx.x == 0;
  if (tr && threadIdx.x == 0) {
    p.trace[kTrTmem] = tmem_base;
    p.trace[kTrNumKb] = static_cast<uint32_t>(num_kb);
  }

  const WaitCtx wprod{abort_flag, p.status, p.wait_limit_ns, kWaitProducer};
  const WaitCtx wmma{abort_flag, p.status, p.wait_limit_ns, kWaitMma};
  const WaitCtx wxf{abort_flag, p.status, p.wait_limit_ns, kWaitTransform};
  const WaitCtx wepi{abort_flag, p.status, p.wait_limit_ns, kWaitEpilogue};

  // MMA completion signals: to this CTA's barrier, or (pair) to the barrier
  // at the same offset in both CTAs.
  auto commit_all = [&](uint64_t* bar) {
    if constexpr (PAIR) {
      umma_commit_pair(in_cta(bar, 0));
      umma_commit_pair(in_cta(bar, 1));
    } else {
      umma_commit(bar);
    }
  };
  // Transform / fold warps report to the MMA issuer (the leader's barrier).
  auto arrive_issuer = [&](uint64_t* bar) {
    if constexpr (PAIR)
      mbar_arrive_cluster(in_cta(bar, 0));
    else
      mbar_arrive(bar);
  };

  // Epilogue helpers of the transform warps: warp w reads TMEM lanes
  // 32 (w % 4).. and column half ((w - 2) / 4) of the tile.
  const int eq = warp & 3;
  const int eh = ((threadIdx.x - 64) >> 5) >> 2;
  const uint32_t e_acc = tmem_base + (static_cast<uint32_t>(eq * 32) << 16) + static_cast<uint32_t>(eh * kHalf);
  const uint32_t e_sum = e_acc + static_cast<uint32_t>(BN);
  const bool no_k = num_kb == 0;  // nothing accumulated: the tile is zero
  // Result columns c .. c+15 of this thread's row: the running sum (chunks
  // [0, nch-1)) + the last chunk's accumulator.
  auto final16 = [&](int c, uint32_t (&r)[16]) {
    if (no_k) {
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = 0u;
      return;
    }
    tmem_ld_32x32b_x16(e_acc + c, r);
    if (SPLIT3 && nch > 1) {
      uint32_t s16[16];
      tmem_ld_32x32b_x16(e_sum + c, s16);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(s16[j]) + __uint_as_float(r[j]));
    } else {
      tmem_wait_ld();
    }
  };
  // Store 16 result columns (col ..) of output row `row` to C (skipped when
  // C is null: a bf16-only intermediate) and its bf16 / lo copies when
  // requested.  Whole 16-column runs go out as 16-byte vectors: a warp's
  // lanes hold 32 different rows, so every store instruction touches 32
  // lines, and scalar 2-byte bf16 stores (16 instructions per run instead
  // of 2) made the epilogue of a bf16-copy product cost most of a tile's MMA time.
  auto store16 = [&](int row, int col, const uint32_t (&r)[16]) {
    if (row >= p.M) return;
    if (p.C != nullptr) {
      const bool vec = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
      float* crow = p.C + static_cast<long long>(row) * p.ldc;
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
    if (p.C_bf16 != nullptr) {
      __nv_bfloat16* brow = p.C_bf16 + static_cast<long long>(row) * p.ldc_bf16;
      const bool bvec = (p.ldc_bf16 % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C_bf16) & 15) == 0);
      if (bvec && col + 16 <= p.N) {
        uint32_t h[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          __nv_bfloat162 t2 = __floats2bfloat162_rn(__uint_as_float(r[2 * v]), __uint_as_float(r[2 * v + 1]));
          h[v] = *reinterpret_cast<uint32_t*>(&t2);
        }
        uint4* dst = reinterpret_cast<uint4*>(brow + col);
        dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
        dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
      } else {
#pragma unroll
        for (int v = 0; v < 16; ++v)
          if (col + v < p.N) brow[col + v] = __float2bfloat16_rn(__uint_as_float(r[v]));
      }
    }
    if (p.C_lo != nullptr) {
      float* lrow = p.C_lo + static_cast<long long>(row) * p.ldc;
#pragma unroll
      for (int v = 0; v < 16; ++v) {
        const float x = __uint_as_float(r[v]);
        if (col + v < p.N) lrow[col + v] = x - tf32_hi(x);
      }
    }
  };
  // Whole-warp stores of 32 result columns through shared memory.  A warp's
  // lanes hold 32 different rows (tensor-memory lane = output row), so a
  // direct store instruction touches 32 rows; transposed through a per-warp
  // 32 x 32 buffer (at wbase, in the then idle stage memory), each store
  // instruction writes four whole 128-byte row segments.  Used once the main
  // loop is done, for fp32 C with 16-byte rows, on whole 32-column runs.
  constexpr int kWs = 36;  // buffer row stride (floats): 16-byte rows, conflict-free quarter-warp phases
  static_assert(8 * 32 * kWs * 4 <= STAGES * kStage, "epilogue transpose buffers fit the stage memory");
  const bool c_vec = p.C != nullptr && (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
  const bool c_plain = c_vec && p.C_bf16 == nullptr && p.C_lo == nullptr;  // nothing but fp32 C to write
  auto store32 = [&](float* wbase, int row0, int col, const uint32_t (&r)[32]) {
    float* wb = wbase + (warp - 2) * 32 * kWs;
    float* mine = wb + lane * kWs;
#pragma unroll
    for (int v = 0; v < 8; ++v)
      reinterpret_cast<float4*>(mine)[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                       __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = j * 32 + lane, rr = i >> 3, c4 = i & 7;
      if (row0 + rr < p.M)
        *reinterpret_cast<float4*>(p.C + static_cast<long long>(row0 + rr) * p.ldc + col + 4 * c4) =
            *reinterpret_cast<const float4*>(wb + rr * kWs + 4 * c4);
    }
    __syncwarp();
  };
  bool acc_valid = false;  // transform warps: the accumulator holds this CTA's result

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, wprod)) break;
        mbar_arrive_expect_tx(&full[s], kTxBytes);
#pragma unroll
        for (int j = 0; j < kSubs; ++j) {
          const int k0 = (kb_begin + i * kSubs + j) * KS;
          if constexpr (kATma) tma_load_2d(a_hi(s) + j * kATileBytes, &tmA, &full[s], k0, m0);
          if constexpr (kBTma) {
#pragma unroll
            for (int c = 0; c < kBCols / MT::kBoxCols; ++c)
              tma_load_2d(b_hi(s) + j * kBTile + c * MT::kBoxBytes, &tmB, &full[s], nb0 + MT::kBoxCols * c, k0);
          }
        }
        ++issued;
      }
      stamp(2);
      if (*abort_flag) {
        // Drain: wait (bounded, ignoring the abort flag) for the last copy
        // issued into each stage, so no bulk copy lands in shared memory
        // after the CTA has exited.
        volatile int no_abort = 0;
        const WaitCtx drain{&no_abort, p.status, p.drain_limit_ns, kWaitDrain};
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; ++i)
          mbar_wait(&full[i % STAGES], (i / STAGES) & 1, drain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The issuing thread is the pipeline's serial step: per stage it only
    // adds small offsets to precomputed descriptor words, tries the stage's
    // barrier once (the slow bounded wait only when it is not ready yet) and
    // commits to precomputed barrier addresses; no 64-bit arithmetic and no
    // divisions in the loop.
    if (lane == 0 && leader) {
      const uint64_t dA0 = make_smem_desc(smem_u32(a_hi(0)), 16, 512, kLayoutSw64);
      const uint64_t dB0 = make_smem_desc(smem_u32(b_hi(0)), MT::kBoxBytes, MT::kBSbo, MT::kBLayout);
      const uint32_t a_lo0 = static_cast<uint32_t>(dA0), a_hi32 = static_cast<uint32_t>(dA0 >> 32);
      const uint32_t b_lo0 = static_cast<uint32_t>(dB0), b_hi32 = static_cast<uint32_t>(dB0 >> 32);
      // Start-address field steps (16-byte units): a k-step along an A row
      // (32 B), along B (kBStepBytes), hi -> lo tile, one stage.
      constexpr uint32_t kAKStep = 32 >> 4, kBKStep = MT::kBStepBytes >> 4;
      constexpr uint32_t kLoOff = (kSubs * (kATileBytes + kBTile)) >> 4;
      constexpr uint32_t kStageOff = kStage >> 4;
      const uint32_t wait0 = smem_u32(kXform ? &ready[0] : &full[0]);
      uint32_t empty_c[PAIR ? 2 : 1], accf_c[PAIR ? 2 : 1];
#pragma unroll
      for (int r = 0; r < (PAIR ? 2 : 1); ++r) {
        empty_c[r] = PAIR ? in_cta(&empty[0], r) : smem_u32(&empty[0]);
        accf_c[r] = PAIR ? in_cta(acc_full, r) : smem_u32(acc_full);
      }
      int s = 0, kc = 0, chunk = 0, issued = 0;
      uint32_t ph = 0, soff = 0;
      for (int i = 0; i < num_kb; ++i) {
        if (!mbar_try_wait(wait0 + 8u * s, ph) && !mbar_wait(kXform ? &ready[s] : &full[s], ph, wmma)) break;
        // 3xTF32: chunk c starts from zero once chunk c-1 has been copied out.
        const bool chunk_start = SPLIT3 ? (kc == 0) : (i == 0);
        if (SPLIT3 && chunk_start && i > 0) {
          if (!mbar_wait(acc_empty, (chunk - 1) & 1, wmma)) break;
        }
        tc_fence_after_sync();
#pragma unroll
        for (int q = 0; q < 2 * kSubs; ++q) {
          // k-step q: block q/2, step q%2.  A: K-major, 64-byte rows, 8-row
          // groups 512 B apart; B: MN-major boxes kBoxBytes apart (LBO),
          // atoms kBSbo apart (SBO).
          const int j = q >> 1, kk = q & 1;
          const uint32_t al = a_lo0 + soff + j * (kATileBytes >> 4) + kk * kAKStep;
          const uint32_t bl = b_lo0 + soff + j * (kBTile >> 4) + kk * kBKStep;
          umma_lohi<PAIR, MT::kBf16>(tmem_base, al, a_hi32, bl, b_hi32, kIdesc, (!chunk_start || q > 0) ? 1u : 0u);
          if constexpr (SPLIT3) {
            umma_lohi<PAIR, false>(tmem_base, al, a_hi32, bl + kLoOff, b_hi32, kIdesc, 1u);
            umma_lohi<PAIR, false>(tmem_base, al + kLoOff, a_hi32, bl, b_hi32, kIdesc, 1u);
          }
        }
#pragma unroll
        for (int r = 0; r < (PAIR ? 2 : 1); ++r) umma_commit_addr<PAIR>(empty_c[r] + 8u * s);
        if constexpr (SPLIT3) {
          if (kc == kChunkS - 1 || i == num_kb - 1) {
#pragma unroll
            for (int r = 0; r < (PAIR ? 2 : 1); ++r) umma_commit_addr<PAIR>(accf_c[r]);
          }
          if (++kc == kChunkS) {
            kc = 0;
            ++chunk;
          }
        }
        ++issued;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
          soff = 0;
        } else {
          soff += kStageOff;
        }
      }
      if (tr) p.trace[kTrMmas] = static_cast<uint32_t>(issued);
      stamp(3);
      // Signals the epilogue; on abort it still fires once every MMA issued
      // so far has finished.  The issuer waits for it too (bounded, ignoring
      // the abort flag) so tensor memory is quiescent before it is freed.
      commit_all(accum_full);
      volatile int no_abort = 0;
      const WaitCtx drain{&no_abort, p.status, p.drain_limit_ns, kWaitDrain};
      mbar_wait(accum_full, 0, drain);
    }
  } else if (warp >= 2 + kXformThreads / 32) {
    // ------------------------------------------------------------ structured-A fill
    if constexpr (kACp) {
      const int ft = threadIdx.x - (64 + kXformThreads);  // 0..kAFillThreads-1
      const int g_first = p.a_row0 + m0;
      for (int i = 0; i < num_kb; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, wprod)) break;
        if constexpr (kStaging) {
          a_stage_fill_toeplitz_bf16<kSubs>(p, stg(s), g_first, (kb_begin + i * kSubs) * KS, ft);
        } else {
#pragma unroll
          for (int j = 0; j < kSubs; ++j)
            a_async_fill<AK>(p, a_hi(s) + j * kATileBytes, g_first, (kb_begin + i * kSubs + j) * KS, ft);
        }
        cp_async_mbar_arrive_noinc(&full[s]);
      }
      // no copy may land after the CTA has exited (bounded: all in flight)
      cp_async_wait_all();
    }
  } else {
    // ------------------------------------------------------------ transform + epilogue
    const int t = threadIdx.x - 64;  // 0..255
    const int xw = t >> 5;           // transform warp 0..7
    const int q = warp & 3;          // TMEM lanes 32q..32q+31 belong to this warp
    const int h = xw >> 2;           // column half of the tile this warp reads back
    const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc_col = tmem_base + lanes + static_cast<uint32_t>(h * kHalf);
    const uint32_t sum_col = acc_col + static_cast<uint32_t>(BN);
    bool ok = true;
    int folded = 0;  // chunks already added into the running sum

    // Add chunk f's accumulator (this warp's 32 lanes x kHalf columns) into
    // the running sum, 32 columns at a time (both loads in flight before one
    // wait, so registers stay few and the MMA waits for 4 round trips, not
    // one per 16 columns), then release the accumulator to the MMA.
    auto fold = [&](int f) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(acc_full, f & 1, wxf))) return false;
      tc_fence_after_sync();
      constexpr int kQ = 32;
#pragma unroll 1
      for (int c0 = 0; c0 < kHalf; c0 += kQ) {
        uint32_t a[kQ], r[kQ];
        tmem_ld_32x32b_x16(acc_col + c0, *reinterpret_cast<uint32_t(*)[16]>(a));
        tmem_ld_32x32b_x16(acc_col + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(a + 16));
        if (f > 0) {
          tmem_ld_32x32b_x16(sum_col + c0, *reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_ld_32x32b_x16(sum_col + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        }
        tmem_wait_ld();
        if (f > 0) {
#pragma unroll
          for (int j = 0; j < kQ; ++j) a[j] = __float_as_uint(__uint_as_float(a[j]) + __uint_as_float(r[j]));
        }
        tmem_st_32x32b_x16(sum_col + c0, *reinterpret_cast<uint32_t(*)[16]>(a));
        tmem_st_32x32b_x16(sum_col + c0 + 16, *reinterpret_cast<uint32_t(*)[16]>(a + 16));
      }
      tmem_wait_st();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) arrive_issuer(acc_empty);
      return true;
    };

    if constexpr (kXform) {
      const int g_first = p.a_row0 + m0;  // structured-A row of this CTA's tile row 0
      // Gathered A values rotate through three register buffers, named at
      // compile time (no register moves): stage i is stored from buffer i % 3
      // while the loads of stage i + 2 are in flight into buffer (i + 2) % 3,
      // so a gather has two stage times to return from L2.
      float a_b0[KS / 2], a_b1[KS / 2], a_b2[KS / 2];
      uint32_t a_rb[KS / 2];
      if constexpr (!kATma && !kACp) {
        a_row_bases<AK, KS>(a_rb, p, g_first, xw, lane);
        if (num_kb > 0) a_gather<AK, KS>(a_b0, p, a_rb, g_first, kb_begin * KS, xw, lane);
        if (num_kb > 1) a_gather<AK, KS>(a_b1, p, a_rb, g_first, (kb_begin + 1) * KS, xw, lane);
      }
      auto stage = [&](int i, const float (&cur)[KS / 2], float (&ahead)[KS / 2]) -> bool {
        const int s = i % STAGES;
        const uint32_t ph = (i / STAGES) & 1;
        // Fold chunk `folded` once the first kFoldLag stages of the next
        // chunk are ready, so the MMA resumes on them as soon as the
        // accumulator is released.  Any lag in [0, STAGES] is deadlock-free
        // (the fold needs only the MMAs of chunk `folded`, whose stages are
        // all ready by now); a lag of STAGES would make the fold wait for a
        // TMA round trip started by the chunk's very last MMA.
        if (SPLIT3 && folded < nch - 1 && i == (folded + 1) * kChunkS + kFoldLag) {
          if (!fold(folded)) return false;
          ++folded;
        }
        if constexpr (!kATma && !kACp) {
          if (i + 2 < num_kb) a_gather<AK, KS>(ahead, p, a_rb, g_first, (kb_begin + i + 2) * KS, xw, lane);
        }
        // Warp-uniform outcome: tcgen05.ld/st are .sync.aligned.
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, wxf))) return false;
        const int k0 = (kb_begin + i * kSubs) * KS;
        // (register-gathered A only with one k-block per stage)
        if constexpr (!kATma && !kACp) a_store<AK, MD>(cur, a_hi(s), a_lo(s), g_first, k0, xw, lane);
        if constexpr (kStaging) {
#pragma unroll
          for (int j = 0; j < kSubs; ++j)
            a_stage_convert_toeplitz_bf16(p, stg(s), a_hi(s) + j * kATileBytes, g_first, k0, j * KS, t);
        }
        if constexpr (!kBTma) {
#pragma unroll 1
          for (int j = 0; j < kSubs; ++j)
            b_build<BK, kBCols, MD>(p, b_hi(s) + j * kBTile, b_lo(s) + j * kBTile, k0 + j * KS, nb0, t);
        }
        if constexpr (SPLIT3) {
          // lo = x - tf32(x) of the TMA-loaded tiles, elementwise at the same
          // (swizzled) offsets.
          auto lo_of = [](const uint8_t* src, uint8_t* dst, int bytes, int tid) {
            const float4* in = reinterpret_cast<const float4*>(src);
            float4* out = reinterpret_cast<float4*>(dst);
#pragma unroll 4
            for (int j = tid; j < bytes / 16; j += kXformThreads) {
              const float4 x = in[j];
              out[j] = make_float4(x.x - tf32_hi(x.x), x.y - tf32_hi(x.y), x.z - tf32_hi(x.z), x.w - tf32_hi(x.w));
            }
          };
          lo_of(a_hi(s), a_lo(s), kSubs * kATileBytes, t);
          if constexpr (kBTma) lo_of(b_hi(s), b_lo(s), kSubs * kBTile, t);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_issuer(&ready[s]);
        return true;
      };
      for (int i = 0; i < num_kb && ok; i += 3) {
        ok = stage(i, a_b0, a_b2);
        if (ok && i + 1 < num_kb) ok = stage(i + 1, a_b1, a_b0);
        if (ok && i + 2 < num_kb) ok = stage(i + 2, a_b2, a_b1);
      }
    }
    if constexpr (SPLIT3) {
      for (; ok && folded < nch - 1; ++folded)
        if (!fold(folded)) ok = false;
    }

    // ------------------------------------------------------------ epilogue
    bool last_ok = ok;
    if (!no_k) {
      if constexpr (SPLIT3)
        last_ok = last_ok && mbar_wait(acc_full, (nch - 1) & 1, wepi);
      else
        last_ok = last_ok && mbar_wait(accum_full, 0, wepi);
    }
    const bool acc_ok = __all_sync(0xffffffffu, last_ok && !*abort_flag);
    acc_valid = acc_ok;
    if (t == 0) stamp(4);
    if (tr && t == 0) p.trace[kTrAccOk] = acc_ok ? 1u : 0u;
    if (SPLITK == 1 && acc_ok) {
      tc_fence_after_sync();
      const int row0 = m0 + q * 32;
#pragma unroll 1
      for (int c = 0; c < kHalf; c += 32) {
        uint32_t r[32];
        final16(c, *reinterpret_cast<uint32_t(*)[16]>(r));
        final16(c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        if (tr && q == 0 && lane == 0 && h == 0 && c == 0)
          for (int j = 0; j < 16; ++j) p.trace[kTrAcc + j] = r[j];
        const int col = n0 + h * kHalf + c;
        if (c_plain && col + 32 <= p.N) {
          store32(reinterpret_cast<float*>(smem), row0, col, r);
        } else {
          store16(row0 + lane, col, *reinterpret_cast<uint32_t(*)[16]>(r));
          store16(row0 + lane, col + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        }
      }
    }
  }

  if constexpr (SPLITK > 1) {
    // Combine the two halves of the K range: CTA 1's results go to CTA 0's
    // stage memory (free once both pipelines are done: every MMA has
    // completed, so every loaded stage was consumed), CTA 0 adds them to its
    // own and stores C.  Both sides move whole rows: CTA 1 transposes each
    // 32 x 32 block through its own buffers so that eight lanes write one
    // 128-byte row segment into CTA 0, and CTA 0 stores its sums the same way
    // (buffers past the exchange tile).  Every thread of both CTAs passes
    // both barriers.
    constexpr int kXld = BN + 4;  // row stride (floats) of the exchange tile: 16-byte rows, few bank conflicts
    static_assert((kBM * kXld + 8 * 32 * kWs) * 4 <= STAGES * kStage,
                  "exchange tile and transpose buffers fit the stage memory");
    float* xbuf = reinterpret_cast<float*>(smem);
    float* wbase = xbuf + kBM * kXld;
    const bool xf = warp >= 2 && warp < 2 + kXformThreads / 32;
    const int xrow = eq * 32 + lane;  // tile row of this transform thread
    tc_fence_before_sync();
    cluster_sync_all();
    tc_fence_after_sync();
    if (xf && krank == 1 && acc_valid) {
      float* wb = wbase + (warp - 2) * 32 * kWs;
      float* mine = wb + lane * kWs;
#pragma unroll 1
      for (int c = 0; c < kHalf; c += 32) {
        uint32_t r[32];
        final16(c, *reinterpret_cast<uint32_t(*)[16]>(r));
        final16(c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
#pragma unroll
        for (int v = 0; v < 8; ++v)
          reinterpret_cast<float4*>(mine)[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                           __uint_as_float(r[4 * v + 2]),
                                                           __uint_as_float(r[4 * v + 3]));
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = j * 32 + lane, rr = i >> 3, c4 = i & 7;
          const float4 v4 = *reinterpret_cast<const float4*>(wb + rr * kWs + 4 * c4);
          const uint32_t dst = mapa_shared(smem_u32(xbuf + (eq * 32 + rr) * kXld + eh * kHalf + c + 4 * c4), 0);
          st_cluster_v4(dst, __float_as_uint(v4.x), __float_as_uint(v4.y), __float_as_uint(v4.z),
                        __float_as_uint(v4.w));
        }
        __syncwarp();
      }
    }
    cluster_sync_all();
    if (threadIdx.x == 64) stamp(5);
    if (xf && krank == 0 && acc_valid) {
#pragma unroll 1
      for (int c = 0; c < kHalf; c += 32) {
        uint32_t r[32];
        final16(c, *reinterpret_cast<uint32_t(*)[16]>(r));
        final16(c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        const float4* src = reinterpret_cast<const float4*>(xbuf + xrow * kXld + eh * kHalf + c);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 o = src[v];
          r[4 * v] = __float_as_uint(__uint_as_float(r[4 * v]) + o.x);
          r[4 * v + 1] = __float_as_uint(__uint_as_float(r[4 * v + 1]) + o.y);
          r[4 * v + 2] = __float_as_uint(__uint_as_float(r[4 * v + 2]) + o.z);
          r[4 * v + 3] = __float_as_uint(__uint_as_float(r[4 * v + 3]) + o.w);
        }
        const int col = n0 + eh * kHalf + c;
        if (c_plain && col + 32 <= p.N) {
          store32(wbase, m0 + eq * 32, col, r);
        } else {
          store16(m0 + xrow, col, *reinterpret_cast<uint32_t(*)[16]>(r));
          store16(m0 + xrow, col + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        }
      }
    }
  }

  tc_fence_before_sync();
  if constexpr (PAIR || SPLITK > 1) {
    // Neither CTA leaves while the leader's MMAs may still read the other's
    // shared memory or the other may still arrive on the leader's barriers
    // (pair), or access the other's shared memory (split).
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  if (threadIdx.x == 64) stamp(7);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace smm
