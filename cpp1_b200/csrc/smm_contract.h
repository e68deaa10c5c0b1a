// Internal interface between the host translation units of libsmm: the
// contraction driver (smm_lib.cu), operand staging and packed-operand
// expansion (smm_stage.cu) and the host-buffer pipeline (smm_host_pipe.cu).
// Not installed; the public interface is include/smm.h.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "smm_host.h"
#include "smm_umma.cuh"

namespace smm {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline size_t round256(size_t b) { return (b + 255) & ~size_t(255); }
inline int round4(int x) { return (x + 3) & ~3; }
inline int round8(int x) { return (x + 7) & ~7; }

bool valid_mode(int mode);

// Packed triangles are addressed with 32-bit offsets on chip.
constexpr int kMaxPackedOrder = 92681;  // N(N+1)/2 < 2^32
int check_packed(const char* who, int N);

// ---------------------------------------------------------------- contraction
// Operand description for run_contraction: a dense TMA-loaded matrix (ptr,
// ld) or a structured one (src, dim, row0).
struct Operand {
  const float* ptr = nullptr;
  const float* lo = nullptr;            // lo plane of ptr (3xTF32), same ld
  const __nv_bfloat16* bf16 = nullptr;  // bf16 copy (bf16 mode), leading dimension ld
  int ld = 0;
  const float* src = nullptr;
  int dim = 0;
  int row0 = 0;
  bool lower = false;  // dense A with exact zeros above the diagonal (K range clipped)
  int tri = 0;         // dense B: 1 upper / 2 lower triangular (K range clipped per column tile)
  // Dense-with-zeros upper-triangular A stacked from row tiles of U (host
  // array of ntiles first rows, tile_rows rows each; see UmmaParams).
  int tile_rows = 0;
  const int* tile_row0 = nullptr;
  int ntiles = 0;
};

Operand dense_op(const float* ptr, const float* lo, int ld, const __nv_bfloat16* bf = nullptr);
Operand structured_op(const float* src, int dim, int row0 = 0);

// Tile choice of one contraction.  Auto sizes the tiles for a launch that
// has the GPU to itself (about a wave of CTAs: narrower tiles, or K split
// over a cluster, when the product is small).  WidePairs always takes 256 x
// 256 CTA-pair tiles (the fastest per flop) when M > 128: for launches that
// share the GPU with other launches of the same call, such as the column
// blocks of a multi-GPU product running side by side.
enum class TilePolicy { Auto, WidePairs };

// C(M x N, ldc) = Aop(M x K) * B(K x N) on stream st.  Optionally also
// writes lo(C) (C_lo, same ldc) or bf16(C) (C_bf16, ldc_bf16) from the
// epilogue, so that C can feed a following product.
int run_contraction(AKind ak, BKind bk, int mode, const Operand& a, const Operand& b, float* C, int ldc, int M,
                    int N, int K, cudaStream_t st, float* C_lo = nullptr, __nv_bfloat16* C_bf16 = nullptr,
                    int ldc_bf16 = 0, TilePolicy policy = TilePolicy::Auto);

// ---------------------------------------------------------------- staging
// A TMA-fed operand (rows x cols row-major): the caller's array or a padded
// copy in the workspace (fp32 modes), or its bf16 copy in the workspace (bf16
// mode).  `lo` stays null: 3xTF32 lo tiles are derived on chip.
struct Staged {
  const float* ptr;
  const float* lo;
  int ld;
  const __nv_bfloat16* bf16 = nullptr;
};

size_t plane_bytes(int rows, int cols);       // fp32 plane, rows padded to 16 bytes
size_t bf16_plane_bytes(int rows, int cols);  // bf16 plane, rows padded to 16 bytes
// Workspace bytes stage_operand takes for this array (0: used in place).
size_t staged_bytes(const float* p, int rows, int cols, int mode);
// The same when the pointer is not known yet (assumes a padded copy).
size_t staged_bytes_bound(int rows, int cols, int mode);
// Stages src (rows x cols, leading dimension cols) for TMA, advancing ws_cur
// past any copy it writes.
int stage_operand(const float* src, int rows, int cols, int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st);

// bf16 copy (round to nearest even) of a rows x cols block of an fp32 matrix
// with leading dimension ld_src (src and ld_src 16-byte aligned for vector
// loads, else scalar) into dst with leading dimension ld_dst (a multiple of
// 8; columns cols .. ld_dst - 1 written as zeros).
int convert_block_bf16(const float* src, int rows, int cols, int ld_src, __nv_bfloat16* dst, int ld_dst,
                       cudaStream_t st);

// Bytes of the dense copy of `rows` rows of a packed operand of order n.
size_t expanded_bytes(int rows, int n, int mode);
// Rows [row0, row0 + rows) of a packed operand (sf: SMM_STRUCT_UPPER, _LOWER
// or _SYMM) as a dense copy (fp32, or bf16 in bf16 mode) at ws_cur.
int expand_operand(const float* P, int sf, int n, int row0, int rows, int mode, uint8_t*& ws_cur, Staged* out,
                   cudaStream_t st);
// Row map of an expansion: slab row r holds matrix row row0[r / tile_rows] +
// r % tile_rows (tile_rows = 0: row0 of the call + r).
struct ExpandRowMap {
  int tile_rows = 0;
  int row0[kMaxMappedTiles] = {};
};
// The same for `rows` rows stacked from ntiles tiles of tile_rows rows (a
// multiple of 64) starting at the matrix rows tile_row0[i]: one launch.
int expand_operand_tiles(const float* P, int sf, int n, const int* tile_row0, int ntiles, int tile_rows, int rows,
                         int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st);
// Bytes of, and the dense copy of, the K x N Toeplitz matrix of generator g
// (K + N - 1 floats; T[k][n] = g[(K-1) + (n-k)]), fp32 or bf16 by mode.
size_t toeplitz_expanded_bytes(int K, int N, int mode);
int expand_toeplitz(const float* g, int K, int N, int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st);
// Whether to expand a packed operand: the workspace holds need_expanded
// bytes and SMM_EXPAND is not 0.
bool expand_packed(void* ws, size_t ws_bytes, size_t need_expanded);

int check_ws(const char* who, void* ws, size_t have, size_t need);
int zero_output(float* C, int rows, int cols, cudaStream_t st);

}  // namespace smm
