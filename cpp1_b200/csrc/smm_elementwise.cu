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
// The symmetric operand is the exception: element (i, j), i > j, lives in
// packed row j, so each CTA takes a pair of mirror tiles, reads their packed
// block once into shared memory and writes both (symm_pair_kernel).
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
  } else if constexpr (SF == SMM_STRUCT_DIAG) {
    return i == j ? __ldg(s + i) : 0.0f;
  } else {  // SMM_STRUCT_TOEPLITZ
    return __ldg(s + (static_cast<long long>(n) - 1 + j - i));
  }
}

// C = A + S (HAS_A) or C = S, all n x n, A and C row-major with leading
// dimension n, S in structured storage of format SF (upper, lower, diagonal,
// Toeplitz: read row-wise, contiguous along j).
template <int SF, bool HAS_A>
__global__ void __launch_bounds__(kEwThreads) dense_struct_kernel(const float* __restrict__ A,
                                                                  const float* __restrict__ S,
                                                                  float* __restrict__ C, int n, int vec) {
  const int row0 = blockIdx.y * kTileR;
  const int col0 = blockIdx.x * kTileC;
  const int t = threadIdx.x;
  const int cq = t & 31;   // column quad
  const int rr = t >> 5;   // row within each group of 8
  const bool below = row0 > col0 + kTileC - 1;       // every i > every j
  const bool above = row0 + kTileR - 1 <= col0;       // every i <= every j
  const bool zero_tile = (SF == SMM_STRUCT_UPPER && below) || (SF == SMM_STRUCT_LOWER && above) ||
                         (SF == SMM_STRUCT_DIAG && (below || above));
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
      s[e] = (j >= n || zero_tile) ? 0.0f : struct_at<SF>(S, n, i, j);
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

// Symmetric operand: one CTA per pair of mirror tiles (I, J), I <= J, of
// kSymT x kSymT.  The packed block P[rows of I][cols of J] (contiguous along
// each packed row) is read once into shared memory, then C[I][J] = A + P and,
// for I != J, C[J][I] = A + P^T are written.  Every packed element crosses
// HBM once (an element-per-output expansion reads the upper triangle twice).
constexpr int kSymT = 64;
constexpr bool kSymPrefetch = false;  // load the dense operand before the barrier

__device__ __forceinline__ void tri_tile(int b, int& I, int& J, int nt) {
  // b enumerates (I, J), I <= J < nt, row by row: row I holds nt - I tiles.
  int lo = 0, hi = nt - 1;
  while (lo < hi) {  // largest I with first(I) <= b, first(I) = I*nt - I(I-1)/2
    const int mid = (lo + hi + 1) >> 1;
    const long long first = static_cast<long long>(mid) * nt - static_cast<long long>(mid) * (mid - 1) / 2;
    if (first <= b) lo = mid; else hi = mid - 1;
  }
  I = lo;
  J = I + static_cast<int>(b - (static_cast<long long>(I) * nt - static_cast<long long>(I) * (I - 1) / 2));
}

template <bool HAS_A>
__global__ void __launch_bounds__(kEwThreads) symm_pair_kernel(const float* __restrict__ A,
                                                               const float* __restrict__ P, float* __restrict__ C,
                                                               int n, int vec) {
  constexpr int T = kSymT;
  constexpr int kQ = T / 4;               // float4 quads per tile row
  constexpr int kRowsPass = kEwThreads / kQ;  // tile rows written per pass
  static_assert(kRowsPass <= T && T % kRowsPass == 0, "tile / thread geometry");
  __shared__ float tile[T][T + 1];
  const int nt = (n + T - 1) / T;
  int I, J;
  tri_tile(blockIdx.x, I, J, nt);
  const int i0 = I * T, j0 = J * T;
  const int t = threadIdx.x;
  const bool pair = I != J;
  const int c4 = 4 * (t % kQ);
  const int rbase = t / kQ;
  // Dense operand of this thread's output quads, loaded before the barrier
  // so the loads overlap the packed-block loads.
  float4 a[2][T / kRowsPass];
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
#pragma unroll
    for (int k = 0; k < T / kRowsPass; ++k) {
      a[tt][k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (HAS_A && kSymPrefetch) {
        const int i = (tt ? j0 : i0) + rbase + kRowsPass * k, j = (tt ? i0 : j0) + c4;
        if (vec && (tt == 0 || pair) && i < n && j + 4 <= n)
          a[tt][k] = __ldcs(reinterpret_cast<const float4*>(A + static_cast<long long>(i) * n + j));
      }
    }
  }
  {
    // packed block rows i (of tile I), columns j (of tile J), i <= j; lanes
    // along j (contiguous in packed row i)
    const int lc = t % T;
#pragma unroll
    for (int k = 0; k < T * T / kEwThreads; ++k) {
      const int lr = t / T + (kEwThreads / T) * k;
      const int i = i0 + lr, j = j0 + lc;
      tile[lr][lc] = (i < n && j < n && i <= j) ? __ldg(P + pk_upper(i, j, n)) : 0.0f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int tt = 0; tt < 2; ++tt) {
    if (tt == 1 && !pair) break;
    const int r0g = tt ? j0 : i0, c0g = tt ? i0 : j0;
#pragma unroll
    for (int k = 0; k < T / kRowsPass; ++k) {
      const int lr = rbase + kRowsPass * k;
      const int i = r0g + lr;
      if (i >= n) continue;
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int lcol = c4 + e;
        if (tt == 0)  // diagonal tiles take the mirror below the diagonal
          v[e] = (!pair && lr > lcol) ? tile[lcol][lr] : tile[lr][lcol];
        else          // C[J rows][I cols] = P^T
          v[e] = tile[lcol][lr];
      }
      const long long base = static_cast<long long>(i) * n;
      const int j = c0g + c4;
      if (vec && j + 4 <= n) {
        float4 c = make_float4(v[0], v[1], v[2], v[3]);
        if constexpr (HAS_A) {
          const float4 x = kSymPrefetch ? a[tt][k] : __ldcs(reinterpret_cast<const float4*>(A + base + j));
          c = make_float4(__fadd_rn(x.x, c.x), __fadd_rn(x.y, c.y), __fadd_rn(x.z, c.z), __fadd_rn(x.w, c.w));
        }
        __stcs(reinterpret_cast<float4*>(C + base + j), c);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (j + e < n) C[base + j + e] = HAS_A ? __fadd_rn(A[base + j + e], v[e]) : v[e];
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

// Packed upper / lower storage from a dense n x n matrix, over the packed
// index: each thread writes 4 consecutive packed elements (one aligned
// 128-bit store when the packed array is 16-byte aligned), reading them from
// the dense row(s) they come from, so reads walk dense rows contiguously and
// writes stream through the packed array.
template <int SF>
__device__ __forceinline__ long long packed_row_start(long long i, long long n) {
  return SF == SMM_STRUCT_LOWER ? i * (i + 1) / 2 : i * n - i * (i - 1) / 2;
}

template <int SF>
__global__ void __launch_bounds__(kEwThreads) pack_kernel(const float* __restrict__ D, float* __restrict__ P,
                                                          int n, int vec) {
  const long long nn = n;
  const long long total = nn * (nn + 1) / 2;
  const long long stride = 4LL * gridDim.x * blockDim.x;
  for (long long p0 = 4LL * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x); p0 < total;
       p0 += stride) {
    // row i holding packed element p0: the largest i with start(i) <= p0
    long long i;
    if constexpr (SF == SMM_STRUCT_LOWER) {
      i = static_cast<long long>((sqrt(8.0 * static_cast<double>(p0) + 1.0) - 1.0) * 0.5);
    } else {
      const double b = 2.0 * static_cast<double>(nn) + 1.0;
      i = static_cast<long long>((b - sqrt(b * b - 8.0 * static_cast<double>(p0))) * 0.5);
    }
    i = i < 0 ? 0 : (i > nn - 1 ? nn - 1 : i);
    while (i > 0 && packed_row_start<SF>(i, nn) > p0) --i;
    while (i + 1 < nn && packed_row_start<SF>(i + 1, nn) <= p0) ++i;
    // column of p0 in row i, then step along the packed order
    long long j = (SF == SMM_STRUCT_LOWER ? 0 : i) + (p0 - packed_row_start<SF>(i, nn));
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[e] = (p0 + e < total) ? __ldcs(D + i * nn + j) : 0.0f;
      ++j;
      const long long row_end = SF == SMM_STRUCT_LOWER ? i + 1 : nn;  // one past the row's last column
      if (j >= row_end) {
        ++i;
        j = SF == SMM_STRUCT_LOWER ? 0 : i;
      }
    }
    if (vec && p0 + 4 <= total) {
      __stcs(reinterpret_cast<float4*>(P + p0), make_float4(v[0], v[1], v[2], v[3]));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (p0 + e < total) P[p0 + e] = v[e];
    }
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
  if (fmt == SMM_STRUCT_SYMM) {
    const long long nt = (n + kSymT - 1) / kSymT;
    const long long pairs = nt * (nt + 1) / 2;
    if (pairs > 0x7FFFFFFFLL) return set_error(SMM_ERR_INVALID, "order %d too large for the tile grid", n);
    symm_pair_kernel<HAS_A><<<static_cast<unsigned>(pairs), kEwThreads, 0, st>>>(A, S, C, n, vec);
    count_launch();
    SMM_CUDA_TRY(cudaGetLastError(), "symmetric elementwise launch");
    return SMM_OK;
  }
  switch (fmt) {
    case SMM_STRUCT_UPPER: dense_struct_kernel<SMM_STRUCT_UPPER, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
    case SMM_STRUCT_LOWER: dense_struct_kernel<SMM_STRUCT_LOWER, HAS_A><<<grid, kEwThreads, 0, st>>>(A, S, C, n, vec); break;
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
  SMM_RANGE("smm_add");
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
  SMM_RANGE("smm_add_struct");
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_add_struct: negative order");
  if (!valid_struct(s_fmt)) return set_error(SMM_ERR_INVALID, "smm_add_struct: unknown structure %d", s_fmt);
  if (N == 0) return SMM_OK;
  if (!A || !S || !C) return set_error(SMM_ERR_INVALID, "smm_add_struct: null pointer");
  if (int rc = launch_dense_struct<true>(A, S, s_fmt, C, N, as_stream(stream))) return rc;
  clear_error();
  return SMM_OK;
}

extern "C" int smm_unpack(const float* S, int s_fmt, float* D, int N, void* stream) {
  SMM_RANGE("smm_unpack");
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_unpack: negative order");
  if (!valid_struct(s_fmt)) return set_error(SMM_ERR_INVALID, "smm_unpack: unknown structure %d", s_fmt);
  if (N == 0) return SMM_OK;
  if (!S || !D) return set_error(SMM_ERR_INVALID, "smm_unpack: null pointer");
  if (int rc = launch_dense_struct<false>(nullptr, S, s_fmt, D, N, as_stream(stream))) return rc;
  clear_error();
  return SMM_OK;
}

extern "C" int smm_pack(const float* D, int s_fmt, float* P, int N, void* stream) {
  SMM_RANGE("smm_pack");
  if (N < 0) return set_error(SMM_ERR_INVALID, "smm_pack: negative order");
  if (s_fmt != SMM_STRUCT_UPPER && s_fmt != SMM_STRUCT_LOWER && s_fmt != SMM_STRUCT_SYMM)
    return set_error(SMM_ERR_INVALID, "smm_pack: structure %d (%s) has no packed triangle", s_fmt,
                     valid_struct(s_fmt) ? struct_name(s_fmt) : "unknown");
  if (N == 0) return SMM_OK;
  if (!D || !P) return set_error(SMM_ERR_INVALID, "smm_pack: null pointer");
  cudaStream_t st = as_stream(stream);
  const long long total = static_cast<long long>(N) * (N + 1) / 2;
  const int grid = grid_for((total + 3) / 4);
  const int vec = aligned16(P) ? 1 : 0;
  if (s_fmt == SMM_STRUCT_LOWER)
    pack_kernel<SMM_STRUCT_LOWER><<<grid, kEwThreads, 0, st>>>(D, P, N, vec);
  else
    pack_kernel<SMM_STRUCT_UPPER><<<grid, kEwThreads, 0, st>>>(D, P, N, vec);
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "smm_pack launch");
  clear_error();
  return SMM_OK;
}

extern "C" int smm_toeplitz_compact(const float* T, float* g, int rows, int cols, void* stream) {
  SMM_RANGE("smm_toeplitz_compact");
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
