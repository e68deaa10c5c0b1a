// Elementwise sums and storage-format converters of the structured formats:
// the DSL's `+` (src/dsl/codegen_cuda.py:1643-1827), packing/expansion of the
// DSL layouts (src/dsl/layout_functions.py:8-68) and the Toeplitz generator
// builder (Cuda kernels/toeplitz.cu:254-261, toeplitz_matmul2.cpp:34-41).
//
// All of it is HBM-bound byte movement with at most one fp32 add per element
// (an IEEE add with one rounding, so results are bit-identical to the
// reference's).  No tensor cores.
//
// Dense x structured kernels work on 32-row x 128-column tiles of the dense
// matrix, 256 threads per CTA, each thread owning a float4 column quad in 4
// rows (128-bit streaming loads/stores of the dense operands when rows are
// 16-byte aligned).  The structured operand is read where it lies: packed rows
// and generator windows are contiguous along j, so lanes along j coalesce.
// The one exception is the mirrored half of a symmetric matrix: element
// (i, j), i > j, lives in packed row j, so a tile wholly below the diagonal is
// read transposed (lanes along i, contiguous in packed row j) into shared
// memory and then consumed row-wise.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "smm_host.h"

namespace smm {
namespace {

constexpr int kTileR = 32;
constexpr int kTileC = 128;
constexpr int kEwThreads = 256;

__device__ __forceinline__ long long pk_upper(long long i, long long j, long long n) {
  return i * n - i * (i - 1) / 2 + (j - i);  // i <= j
}
__device__ __forceinline__ long long pk_lower(long long i, long long j) {
  return i * (i + 1) / 2 + j;  // j <= i
}

// Value of the expanded structured operand at (i, j), both inside [0, n).
template <int SF>
__device__ __forceinline__ float struct_at(const float* __restrict__ s, int n, int i, int j) {
  if constexpr (SF == SMM_STRUCT_UPPER) {
    return i <= j ? __ldg(s + pk_upper(i, j, n)) : 0.0f;
  } else if constexpr (SF == SMM_STRUCT_LOWER) {
    return j <= i ? __ldg(s + pk_lower(i, j)) : 0.0f;
  } else if constexpr (SF == SMM_STRUCT_SYMM) {
    return i <= j ? __ldg(s + pk_upper(i, j, n)) : __ldg(s + pk_upper(j, i, n));
  } else if constexpr (SF == SMM_STRUCT_DIAG) {
    return i == j ? __ldg(s + i) : 0.0f;
  } else {  // SMM_STRUCT_TOEPLITZ
    return __ldg(s + (static_cast<long long>(n) - 1 + j - i));
  }
}

// C = A + S (HAS_A) or C = S, all n x n, A and C row-major with leading
// dimension n, S in structured storage of format SF.
template <int SF, bool HAS_A>
__global__ void __launch_bounds__(kEwThreads) dense_struct_kernel(const float* __restrict__ A,
                                                                  const float* __restrict__ S,
                                                                  float* __restrict__ C, int n, int vec) {
  __shared__ float tr[kTileR][kTileC + 1];  // transposed staging (symmetric, below the diagonal)
  const int row0 = blockIdx.y * kTileR;
  const int col0 = blockIdx.x * kTileC;
  const int t = threadIdx.x;
  const int cq = t & 31;   // column quad
  const int rr = t >> 5;   // row within each group of 8
  const bool below = row0 > col0 + kTileC - 1;       // every i > every j
  const bool above = row0 + kTileR - 1 <= col0;       // every i <= every j
  const bool zero_tile = (SF == SMM_STRUCT_UPPER && below) || (SF == SMM_STRUCT_LOWER && above) ||
                         (SF == SMM_STRUCT_DIAG && (below || above));
  const bool staged = (SF == SMM_STRUCT_SYMM) && below;
  if (staged) {
    // element (i, j) = S[j][i], packed row j: lanes along i
    const int li = t & 31;
#pragma unroll 4
    for (int k = 0; k < kTileC / 8; ++k) {
      const int lj = (t >> 5) + 8 * k;
      const int i = row0 + li, j = col0 + lj;
      tr[li][lj] = (i < n && j < n) ? __ldg(S + pk_upper(j, i, n)) : 0.0f;
    }
    __syncthreads();
  }
#pragma unroll
  for (int it = 0; it < kTileR / 8; ++it) {
    const int r = rr + 8 * it;
    const int i = row0 + r;
    if (i >= n) break;
    const int j0 = col0 + 4 * cq;
    if (j0 >= n) continue;
    const long long base = static_cast<long long>(i) * n;
    float s[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = j0 + e;
      if (j >= n || zero_tile) {
        s[e] = 0.0f;
      } else if (staged) {
        s[e] = tr[r][4 * cq + e];
      } else {
        s[e] = struct_at<SF>(S, n, i, j);
      }
    }
    if (vec && j0 + 4 <= n) {
      float4 c = make_float4(s[0], s[1], s[2], s[3]);
      if constexpr (HAS_A) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(A + base + j0));
        c = make_float4(__fadd_rn(a.x, c.x), __fadd_rn(a.y, c.y), __fadd_rn(a.z, c.z), __fadd_rn(a.w, c.w));
      }
      __stcs(reinterpret_cast<float4*>(C + base + j0), c);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = j0 + e;
        if (j < n) C[base + j] = HAS_A ? __fadd_rn(A[base + j], s[e]) : s[e];
      }
    }
  }
}

// C[k] = A[k] + B[k], k < count: 128-bit path over the 16-byte-aligned body.
__global__ void __launch_bounds__(kEwThreads) add_vec4_kernel(const float4* __restrict__ A,
                                                              const float4* __restrict__ B, float4* __restrict__ C,
                                                              long long n4) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < n4; k += stride) {
    const float4 a = __ldcs(A + k), b = __ldcs(B + k);
    __stcs(C + k, make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w)));
  }
}
__global__ void __launch_bounds__(kEwThreads) add_scalar_kernel(const float* __restrict__ A,
                                                                const float* __restrict__ B, float* __restrict__ C,
                                                                long long count) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < count; k += stride)
    C[k] = __fadd_rn(A[k], B[k]);
}

// Packed upper / lower storage from a dense n x n matrix: block (x, i) copies
// chunk x (1024 elements) of packed row i.
template <int SF>
__global__ void __launch_bounds__(kEwThreads) pack_kernel(const float* __restrict__ D, float* __restrict__ P,
                                                          int n) {
  const int i = blockIdx.y;
  const int len = (SF == SMM_STRUCT_LOWER) ? i + 1 : n - i;  // packed row length
  const int first = (SF == SMM_STRUCT_LOWER) ? 0 : i;          // first dense column
  const long long out0 = (SF == SMM_STRUCT_LOWER) ? pk_lower(i, 0) : pk_upper(i, i, n);
  const float* src = D + static_cast<long long>(i) * n + first;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int k = blockIdx.x * (4 * kEwThreads) + e * kEwThreads + threadIdx.x;
    if (k < len) P[out0 + k] = __ldcs(src + k);
  }
}

// Generator g[rows + cols - 1] of a rows x cols Toeplitz matrix T:
// g[rows-1-i] = T[i][0], g[rows-1+j] = T[0][j].
__global__ void __launch_bounds__(kEwThreads) toeplitz_compact_kernel(const float* __restrict__ T,
                                                                      float* __restrict__ g, int rows, int cols) {
  const long long total = static_cast<long long>(rows) + cols - 1;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long k = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; k < total; k += stride) {
    if (k < rows) {
      const long long i = rows - 1 - k;  // first column, reversed
      g[k] = T[i * cols];
    } else {
      g[k] = T[k - (rows - 1)];  // first row, j >= 1
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool valid_struct(int f) { return f >= SMM_STRUCT_UPPER && f <= SMM_STRUCT_TOEPLITZ; }
const char* struct_name(int f) {
  switch (f) {
    case SMM_STRUCT_UPPER: return "upper";
    case SMM_STRUCT_LOWER: return "lower";
    case SMM_STRUCT_SYMM: return "symmetric";
    case SMM_STRUCT_DIAG: return "diagonal";
    default: return "toeplitz";
  }
}

template <bool HAS_A>
int launch_dense_struct(const float* A, const float* S, int fmt, float* C, int n, cudaStream_t st) {
  const dim3 grid((n + kTileC - 1) / kTileC, (n + kTileR - 1) / kTileR);
  if (grid.y > 65535u) return set_error(SMM_ERR_INVALID, "order %d too large for the tile grid", n);
  const int vec = (n % 4 == 0) && aligned16(C) && (!HAS_A || aligned16(A)) ? 1 : 0;
  switch (fmt) {
    case SMM_STRUCT_UPPER: dense_struct_kernel<SMM_STRUCT_UPPER, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
    case SMM_STRUCT_LOWER: dense_struct_kernel<SMM_STRUCT_LOWER, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
    case SMM_STRUCT_SYMM: dense_struct_kernel<SMM_STRUCT_SYMM, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
    case SMM_STRUCT_DIAG: dense_struct_kernel<SMM_STRUCT_DIAG, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
    default: dense_struct_kernel<SMM_STRUCT_TOEPLITZ, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
  }
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "dense x structured elementwise launch");
  return SMM_OK;
}

int grid_for(long long work) {
  return static_cast<int>(std::max<long long>(1, std::min<long long>((work + kEwThreads - 1) / kEwThreads, 148LL * 16)));
}

}  // namespace
}  // namespace smm

using namespace smm;

extern "C" int smm_add(const float* A, const float* B, float* C, long long count, void* stream) {
  if (count < 0) return set_error(SMM_ERR_INVALID, "smm_add: negative count");
  if (count == 0) return SMM_OK;
  if (!A || !B || !C) return set_error(SMM_ERR_INVALID, "smm_add: null pointer");
  cudaStream_t st = as_stream(stream);
  long long done = 0;
  if (aligned16(A) && aligned16(B) && aligned16(C)) {
    const long long n4 = count / 4;
    if (n4 > 0) {
      add_vec4_kernel<<<grid_for(n4), kEwThreads, 0, st>>>(reinterpret_cast<const float4*>(A),
                                                            reinterpret_cast<const float4*>(B),
                                                            reinterpret_cast<float4*>(C), n4);
      count_launch();
      SMM_CUDA_TRY(cudaGetLastError(), "smm_add launch");
    }
    done = 4 * n4;
  }
  if (done < count) {
    add_scalar_kernel<<<grid_for(count - done), kEwThreads, 0, st>>>(A + done, B + done, C + done, count - done);
    count_launch();
    SMM_CUDA_TRY(cudaGetLastError(), "smm_add launch");
  }
  clear_error();
  return SMM_OK;
}

extern "C" int smm_add_struct(const float* A, const float* S, int s_fmt, float* C, int N, void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_add_struct: negative order");
  if (!valid_struct(s_fmt)) return set_error(SMM_ERR_INVALID, "smm_add_struct: unknown structure %d", s_fmt);
  if (N == 0) return SMM_OK;
  if (!A || !S || !C) return set_error(SMM_ERR_INVALID, "smm_add_struct: null pointer");
  if (int rc = launch_dense_struct<true>(A, S, s_fmt, C, N, as_stream(stream))) return rc;
  clear_error();
  return SMM_OK;
}

extern "C" int smm_unpack(const float* S, int s_fmt, float* D, int N, void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_unpack: negative order");
  if (!valid_struct(s_fmt)) return set_error(SMM_ERR_INVALID, "smm_unpack: unknown structure %d", s_fmt);
  if (N == 0) return SMM_OK;
  if (!S || !D) return set_error(SMM_ERR_INVALID, "smm_unpack: null pointer");
  if (int rc = launch_dense_struct<false>(nullptr, S, s_fmt, D, N, as_stream(stream))) return rc;
  clear_error();
  return SMM_OK;
}

extern "C" int smm_pack(const float* D, int s_fmt, float* P, int N, void* stream) {
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_pack: negative order");
  if (s_fmt != SMM_STRUCT_UPPER && s_fmt != SMM_STRUCT_LOWER && s_fmt != SMM_STRUCT_SYMM)
    return set_error(SMM_ERR_INVALID, "smm_pack: structure %d (%s) has no packed triangle", s_fmt,
                     valid_struct(s_fmt) ? struct_name(s_fmt) : "unknown");
  if (N == 0) return SMM_OK;
  if (!D || !P) return set_error(SMM_ERR_INVALID, "smm_pack: null pointer");
  if (N > 65535) return set_error(SMM_ERR_INVALID, "smm_pack: order %d above 65535", N);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((N + 4 * kEwThreads - 1) / (4 * kEwThreads), N);
  if (s_fmt == SMM_STRUCT_LOWER)
    pack_kernel<SMM_STRUCT_LOWER><<<grid, kEwThreads, 0, st>>>(D, P, N);
  else
    pack_kernel<SMM_STRUCT_UPPER><<<grid, kEwThreads, 0, st>>>(D, P, N);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "smm_pack launch");
  clear_error();
  return SMM_OK;
}

extern "C" int smm_toeplitz_compact(const float* T, float* g, int rows, int cols, void* stream) {
  if (rows < 0 || cols < 0) return set_error(SMM_ERR_INVALID, "smm_toeplitz_compact: negative shape");
  if (rows == 0 || cols == 0) return SMM_OK;
  if (!T || !g) return set_error(SMM_ERR_INVALID, "smm_toeplitz_compact: null pointer");
  cudaStream_t st = as_stream(stream);
  const long long total = static_cast<long long>(rows) + cols - 1;
  toeplitz_compact_kernel<<<grid_for(total), kEwThreads, 0, st>>>(T, g, rows, cols);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "smm_toeplitz_compact launch");
  clear_error();
  return SMM_OK;
}
