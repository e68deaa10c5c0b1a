// Operand staging for the tensor-core contractions: padded fp32 copies and
// bf16 copies of dense operands (TMA needs 16-byte row strides), and the
// dense expansion of packed upper / lower / symmetric operands.  All of it
// is HBM-bound copying inside the product call.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "smm_contract.h"
#include "smm_device.cuh"
#include "smm_host.h"

namespace smm {
namespace {

// dst = src with zero columns appended up to ld_dst (a multiple of 4), so
// that TMA can address its rows.  The source is unaligned or has rows that
// are not 16-byte multiples (else it is used in place), so each thread reads
// 4 consecutive elements of a row with scalar loads and writes them with one
// 128-bit store.  Blocks run along a row (x) and stride over rows (y).
__global__ void __launch_bounds__(256) pad_rows_kernel(const float* __restrict__ src, int rows, int cols,
                                                       int ld_src, float* __restrict__ dst, int ld_dst) {
  const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= ld_dst) return;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const float* s = src + static_cast<long long>(r) * ld_src + c;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = c + e < cols ? __ldcs(s + e) : 0.0f;
    *reinterpret_cast<float4*>(dst + static_cast<long long>(r) * ld_dst + c) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// bf16 copy of an fp32 matrix (round to nearest even), rows padded with zeros
// to ld_dst elements (a multiple of 8).  Each thread converts 8 consecutive
// elements of a row: two 128-bit streaming loads when the source rows are
// 16-byte aligned (vec), one 128-bit store.  Blocks run along a row (x) and
// stride over rows (y); no per-element index division.
__global__ void __launch_bounds__(256) to_bf16_kernel(const float* __restrict__ src, int rows, int cols, int ld_src,
                                                      __nv_bfloat16* __restrict__ dst, int ld_dst, int vec) {
  const int c = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= ld_dst) return;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const float* s = src + static_cast<long long>(r) * ld_src + c;
    float v[8];
    if (vec && c + 8 <= cols) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(s));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(s + 4));
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = c + e < cols ? s[e] : 0.0f;
    }
    uint4 o;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]), h3 = __floats2bfloat162_rn(v[6], v[7]);
    o.x = *reinterpret_cast<uint32_t*>(&h0);
    o.y = *reinterpret_cast<uint32_t*>(&h1);
    o.z = *reinterpret_cast<uint32_t*>(&h2);
    o.w = *reinterpret_cast<uint32_t*>(&h3);
    *reinterpret_cast<uint4*>(dst + static_cast<long long>(r) * ld_dst + c) = o;
  }
}

bool needs_pad(const float* p, int cols) { return (cols % 4 != 0) || !aligned16(p); }
// Dense copy (fp32, or bf16 rounded to nearest even) of rows [row0, row0 +
// rows) of a packed structured matrix of order n: upper (zeros below the
// diagonal), lower (zeros above) or symmetric (mirrored), each row padded with
// zeros to ld (even).  64 x 64 tiles, 256 threads, lanes along columns (two
// per lane: coalesced packed-row reads and row writes).  A symmetric tile
// wholly below the diagonal holds mirrors S[j][i]: it reads its block along
// packed rows j (coalesced) and transposes it through shared memory.
__device__ __forceinline__ void store_pair(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void store_pair(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
template <int SF, typename T>
__global__ void __launch_bounds__(256) expand_kernel(const float* __restrict__ P, int n, int row0, int rows,
                                                     T* __restrict__ dst, int ld, uint32_t* status,
                                                     const ExpandRowMap map) {
  const long long len = static_cast<long long>(n) * (n + 1) / 2;
  __shared__ float tile[64][65];
  const int r0 = blockIdx.y * 64;  // slab row of the tile
  const int c0 = blockIdx.x * 64;  // column of the tile
  const int t = threadIdx.x;
  // matrix row of slab row r0 (the 64-row tile lies inside one mapped tile)
  const int g0 = map.tile_rows > 0 ? map.row0[r0 / map.tile_rows] + r0 % map.tile_rows : row0 + r0;
  const bool mirror = SF == SMM_STRUCT_SYMM && c0 + 63 < g0;
  if (mirror) {
    const int il = t & 63;
    const int i = g0 + il;
    for (int jl = t >> 6; jl < 64; jl += 4) {
      const int j = c0 + jl;  // j < i for every element of the tile
      tile[jl][il] = (r0 + il < rows && j < n) ? ld_chk(P, packed_idx(j, i, n), len, status, kBoundsExpand) : 0.0f;
    }
    __syncthreads();
  }
  const int cp = 2 * (t & 31);
  const int j = c0 + cp;
  if (j >= ld) return;  // ld and j even: both columns of the pair are inside or outside
  for (int rl = t >> 5; rl < 64; rl += 8) {
    const int r = r0 + rl;
    if (r >= rows) break;
    const int i = g0 + rl;
    float v[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int jj = j + e;
      if (mirror) {
        v[e] = tile[cp + e][rl];
      } else if (jj >= n) {
        v[e] = 0.0f;
      } else if constexpr (SF == SMM_STRUCT_UPPER) {
        v[e] = jj >= i ? ld_chk(P, packed_idx(i, jj, n), len, status, kBoundsExpand) : 0.0f;
      } else if constexpr (SF == SMM_STRUCT_LOWER) {
        v[e] = jj <= i ? ld_chk(P, static_cast<long long>(i) * (i + 1) / 2 + jj, len, status, kBoundsExpand) : 0.0f;
      } else {
        v[e] = ld_chk(P, jj >= i ? packed_idx(i, jj, n) : packed_idx(jj, i, n), len, status, kBoundsExpand);
      }
    }
    store_pair(dst + static_cast<long long>(r) * ld + j, v[0], v[1]);
  }
}

// Dense copy of the K x N Toeplitz matrix of generator g (K + N - 1 floats),
// T[k][n] = g[(K-1) + (n-k)]: row k is the window g[K-1-k ..].  Threads write
// column pairs of a row (coalesced window reads and row writes); blocks run
// along a row (x) and stride over rows (y).  Columns N .. ld-1 are zero.
template <typename T>
__global__ void __launch_bounds__(256) toeplitz_expand_kernel(const float* __restrict__ g, int K, int N,
                                                              T* __restrict__ dst, int ld, uint32_t* status) {
  const int j = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (j >= ld) return;
  const long long len = static_cast<long long>(K) + N - 1;
  for (int k = blockIdx.y; k < K; k += gridDim.y) {
    const long long w = K - 1 - k;
    const float a = j < N ? ld_chk(g, w + j, len, status, kBoundsExpand) : 0.0f;
    const float b = j + 1 < N ? ld_chk(g, w + j + 1, len, status, kBoundsExpand) : 0.0f;
    store_pair(dst + static_cast<long long>(k) * ld + j, a, b);
  }
}

template <typename T>
void launch_expand(const float* P, int sf, int n, int row0, int rows, T* dst, int ld, cudaStream_t st,
                   const ExpandRowMap& map = ExpandRowMap{}) {
  const dim3 grid((ld + 63) / 64, (rows + 63) / 64);
  switch (sf) {
    case SMM_STRUCT_UPPER:
      expand_kernel<SMM_STRUCT_UPPER, T><<<grid, 256, 0, st>>>(P, n, row0, rows, dst, ld, device_status_word(), map);
      break;
    case SMM_STRUCT_LOWER:
      expand_kernel<SMM_STRUCT_LOWER, T><<<grid, 256, 0, st>>>(P, n, row0, rows, dst, ld, device_status_word(), map);
      break;
    default:
      expand_kernel<SMM_STRUCT_SYMM, T><<<grid, 256, 0, st>>>(P, n, row0, rows, dst, ld, device_status_word(), map);
      break;
  }
}

}  // namespace

size_t plane_bytes(int rows, int cols) { return round256(static_cast<size_t>(rows) * round4(cols) * sizeof(float)); }
size_t bf16_plane_bytes(int rows, int cols) { return round256(static_cast<size_t>(rows) * round8(cols) * 2); }
size_t staged_bytes(const float* p, int rows, int cols, int mode) {
  if (mode == SMM_MODE_BF16) return bf16_plane_bytes(rows, cols);
  return needs_pad(p, cols) ? plane_bytes(rows, cols) : 0;
}
// Workspace bound when the pointer is not known yet (assumes a padded copy).
size_t staged_bytes_bound(int rows, int cols, int mode) {
  if (mode == SMM_MODE_BF16) return bf16_plane_bytes(rows, cols);
  return plane_bytes(rows, cols);
}

int convert_block_bf16(const float* src, int rows, int cols, int ld_src, __nv_bfloat16* dst, int ld_dst,
                       cudaStream_t st) {
  if (rows <= 0 || ld_dst <= 0) return SMM_OK;
  const int gx = (ld_dst / 8 + 255) / 256;
  const int gy = std::max(1, std::min(rows, std::max(1, 148 * 16 / gx)));
  const int vec = (ld_src % 4 == 0 && aligned16(src)) ? 1 : 0;
  to_bf16_kernel<<<dim3(gx, gy), 256, 0, st>>>(src, rows, cols, ld_src, dst, ld_dst, vec);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "bf16 block conversion launch");
  return SMM_OK;
}

int stage_operand(const float* src, int rows, int cols, int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st) {
  if (mode == SMM_MODE_BF16) {
    const int ld = round8(cols);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ws_cur);
    ws_cur += bf16_plane_bytes(rows, cols);
    const int gx = (ld / 8 + 255) / 256;
    const int gy = std::max(1, std::min(rows, std::max(1, 148 * 16 / gx)));
    const int vec = (cols % 4 == 0 && aligned16(src)) ? 1 : 0;
    to_bf16_kernel<<<dim3(gx, gy), 256, 0, st>>>(src, rows, cols, cols, dst, ld, vec);
    count_launch();
    SMM_CUDA_TRY(cudaGetLastError(), "bf16 staging launch");
    *out = {nullptr, nullptr, ld, dst};
    return SMM_OK;
  }
  // fp32 modes: the caller's array when TMA can address it (the 3xTF32 lo
  // tiles are derived on chip), else a copy with 16-byte-multiple rows.
  if (!needs_pad(src, cols)) {
    *out = {src, nullptr, cols};
    return SMM_OK;
  }
  const int ld = round4(cols);
  float* dst = reinterpret_cast<float*>(ws_cur);
  ws_cur += plane_bytes(rows, cols);
  const int gx = (ld / 4 + 255) / 256;
  const int gy = std::max(1, std::min(rows, std::max(1, 148 * 16 / gx)));
  pad_rows_kernel<<<dim3(gx, gy), 256, 0, st>>>(src, rows, cols, cols, dst, ld);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "operand staging launch");
  *out = {dst, nullptr, ld};
  return SMM_OK;
}

// A packed operand (upper, lower or symmetric) on the left: rows [row0, row0 +
// rows) expanded into a dense copy in the workspace (fp32 in the fp32 modes,
// bf16 in bf16 mode), which the tensor cores then read by TMA like any dense
// operand.  A packed row has no fixed alignment, so an on-chip fill of it
// issues one 4-byte copy per element; the expansion is one HBM pass that
// costs ~3% of the product at N = 4096..8192 (measured with it: U B 3xTF32
// 218 -> 258 TFLOP/s, TF32 258 -> 569; S B 3xTF32 158 -> 200).
size_t expanded_bytes(int rows, int n, int mode) {
  return mode == SMM_MODE_BF16 ? bf16_plane_bytes(rows, n) : plane_bytes(rows, n);
}
int expand_operand(const float* P, int sf, int n, int row0, int rows, int mode, uint8_t*& ws_cur, Staged* out,
                   cudaStream_t st) {
  if (mode == SMM_MODE_BF16) {
    const int ld = round8(n);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ws_cur);
    launch_expand(P, sf, n, row0, rows, dst, ld, st);
    *out = {nullptr, nullptr, ld, dst};
  } else {
    const int ld = round4(n);
    float* dst = reinterpret_cast<float*>(ws_cur);
    launch_expand(P, sf, n, row0, rows, dst, ld, st);
    *out = {dst, nullptr, ld};
  }
  ws_cur += expanded_bytes(rows, n, mode);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "packed operand expansion launch");
  return SMM_OK;
}

int expand_operand_tiles(const float* P, int sf, int n, const int* tile_row0, int ntiles, int tile_rows, int rows,
                         int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st) {
  if (ntiles < 1 || ntiles > kMaxMappedTiles || tile_rows < 64 || tile_rows % 64 != 0 ||
      static_cast<long long>(ntiles) * tile_rows < rows)
    return set_error(SMM_ERR_INVALID, "internal: bad expansion row map (%d tiles of %d rows for %d rows)", ntiles,
                     tile_rows, rows);
  ExpandRowMap map;
  map.tile_rows = tile_rows;
  for (int i = 0; i < ntiles; ++i) map.row0[i] = tile_row0[i];
  if (mode == SMM_MODE_BF16) {
    const int ld = round8(n);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ws_cur);
    launch_expand(P, sf, n, 0, rows, dst, ld, st, map);
    *out = {nullptr, nullptr, ld, dst};
  } else {
    const int ld = round4(n);
    float* dst = reinterpret_cast<float*>(ws_cur);
    launch_expand(P, sf, n, 0, rows, dst, ld, st, map);
    *out = {dst, nullptr, ld};
  }
  ws_cur += expanded_bytes(rows, n, mode);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "packed operand expansion launch");
  return SMM_OK;
}

size_t toeplitz_expanded_bytes(int K, int N, int mode) {
  return mode == SMM_MODE_BF16 ? bf16_plane_bytes(K, N) : plane_bytes(K, N);
}
int expand_toeplitz(const float* g, int K, int N, int mode, uint8_t*& ws_cur, Staged* out, cudaStream_t st) {
  const bool bf = mode == SMM_MODE_BF16;
  const int ld = bf ? round8(N) : round4(N);
  const int gx = (ld / 2 + 255) / 256;
  const int gy = std::max(1, std::min(K, std::max(1, 148 * 16 / gx)));
  if (bf) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ws_cur);
    toeplitz_expand_kernel<__nv_bfloat16><<<dim3(gx, gy), 256, 0, st>>>(g, K, N, dst, ld, device_status_word());
    *out = {nullptr, nullptr, ld, dst};
  } else {
    float* dst = reinterpret_cast<float*>(ws_cur);
    toeplitz_expand_kernel<float><<<dim3(gx, gy), 256, 0, st>>>(g, K, N, dst, ld, device_status_word());
    *out = {dst, nullptr, ld};
  }
  ws_cur += toeplitz_expanded_bytes(K, N, mode);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "Toeplitz expansion launch");
  return SMM_OK;
}

// Expand a packed left operand when the workspace has room for the copy (the
// *_workspace_size functions include it); a smaller workspace (down to what
// the on-chip path needs) builds the operand on chip instead.  SMM_EXPAND=0
// forces the on-chip path.
bool expand_packed(void* ws, size_t ws_bytes, size_t need_expanded) {
  const char* e = std::getenv("SMM_EXPAND");
  if (e && e[0] == '0') return false;
  return ws != nullptr && ws_bytes >= need_expanded;
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

}  // namespace smm
