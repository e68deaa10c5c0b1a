/* CPU oracle for the structured matrix-multiply path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the library (cpp1_b200/) links, loads
 * or calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline use it, as the checker.
 *
 * Two families of functions:
 *
 *  1. fp32 restatements of the reference's CPU kernels.  Every reference
 *     kernel (gemm_benchmark.cpp:40-156, upper_triag_matmul.cpp:41-137,
 *     symmetric_matmul.cpp:84-211, toeplitz_matmul2.cpp:44-144) keeps one
 *     fp32 accumulator per output element, initialised from C (zero), and
 *     updates it with one fused multiply-add per k (_mm256_fmadd_ps), k in
 *     ascending order across and within K-blocks.  Restated with fmaf in the
 *     same order, the results are bit-identical to the compiled reference
 *     kernels (checked against them by the golden fixtures).  For the
 *     left-side operations the order is that of the exact permutation the
 *     reference is run through (see each function).
 *     The diagonal scale (diag_matmul.cpp:45-111) is one fp32 multiply.
 *
 *  2. fp64 ground truth on a list of output rows, used to measure normwise
 *     relative error at sizes where a full recomputation is too slow.
 *
 * Storage conventions (all row-major fp32):
 *   packed upper / symmetric: idx(i,j) = i*N - i(i-1)/2 + (j-i), i <= j,
 *     length N(N+1)/2 (src/dsl/layout_functions.py:8-23, 50-68);
 *   Toeplitz generator g[2N-1]: T[i][j] = g[(N-1) + (j-i)]
 *     (src/dsl/layout_functions.py:45-48; toeplitz_matmul2.cpp:35-42).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline size_t pidx(long i, long j, long n) { return (size_t)(i * n - i * (i - 1) / 2 + (j - i)); }

/* S[i][j] from packed upper storage, mirrored below the diagonal
 * (symmetric_matmul.cpp:47-50 get_symmetric_compact_element). */
static inline float sym_at(const float* Sp, long i, long j, long n) {
  return i <= j ? Sp[pidx(i, j, n)] : Sp[pidx(j, i, n)];
}

/* ---------------- fp32 restatements ---------------- */

/* C(MxN) = A(MxK) B(KxN); gemm_benchmark.cpp:40-156. */
void orc_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < M; ++i) {
    float* c = C + (size_t)i * N;
    for (long j = 0; j < N; ++j) c[j] = 0.0f;
    for (long k = 0; k < K; ++k) {
      const float a = A[(size_t)i * K + k];
      const float* b = B + (size_t)k * N;
      for (long j = 0; j < N; ++j) c[j] = fmaf(a, b[j], c[j]);
    }
  }
}

/* C[i][j] = d[i] * B[i][j]; one rounding (diag_matmul.cpp:45-111 applied to
 * the transpose, and src/dsl/codegen_cuda.py:1275-1307 kernel_diag_x_gen). */
void orc_diag_rows_f32(const float* d, const float* B, float* C, int M, int N) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < M; ++i) {
    const float s = d[i];
    for (long j = 0; j < N; ++j) C[(size_t)i * N + j] = s * B[(size_t)i * N + j];
  }
}

/* C[i][j] = A[i][j] * b[j]; diag_matmul.cpp:45-111 as the driver runs it. */
void orc_diag_cols_f32(const float* A, const float* b, float* C, int M, int N) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < M; ++i)
    for (long j = 0; j < N; ++j) C[(size_t)i * N + j] = A[(size_t)i * N + j] * b[j];
}

/* C(N x ncols) = U(N x N, packed upper) B(N x ncols).
 * The reference computes only A*U (upper_triag_matmul.cpp:41-137); C = U*B
 * is run through it as (U B)^T = (B^T J)(J U^T J) J, whose ascending k
 * becomes, for C[c][r], the terms U[c][k] B[k][r] accumulated from k = N-1
 * down to k = c. */
void orc_upper_left_f32(const float* Up, const float* B, float* C, int N, int ncols) {
  const long n = N;
#pragma omp parallel for schedule(dynamic, 4)
  for (long c = 0; c < n; ++c) {
    float* out = C + (size_t)c * ncols;
    for (long r = 0; r < ncols; ++r) out[r] = 0.0f;
    for (long k = n - 1; k >= c; --k) {
      const float u = Up[pidx(c, k, n)];
      const float* b = B + (size_t)k * ncols;
      for (long r = 0; r < ncols; ++r) out[r] = fmaf(b[r], u, out[r]);
    }
  }
}

/* Y(MxN) = X(MxN) U(NxN packed upper); upper_triag_matmul.cpp:41-137 as the
 * driver runs it (terms with k > j are exact zeros and leave the sum alone). */
void orc_upper_right_f32(const float* X, const float* Up, float* Y, int M, int N) {
  const long n = N;
#pragma omp parallel for schedule(static)
  for (long i = 0; i < M; ++i) {
    float* y = Y + (size_t)i * n;
    for (long j = 0; j < n; ++j) y[j] = 0.0f;
    for (long k = 0; k < n; ++k) {
      const float a = X[(size_t)i * n + k];
      const float* urow = Up + pidx(k, k, n) - k; /* urow[j] = U[k][j] for j >= k */
      for (long j = k; j < n; ++j) y[j] = fmaf(a, urow[j], y[j]);
    }
  }
}

/* W(MxN) = A(MxN) S(NxN packed upper, symmetric); symmetric_matmul.cpp:84-211. */
void orc_symm_right_f32(const float* A, const float* Sp, float* W, int M, int N) {
  const long n = N;
  float* srow = (float*)malloc(sizeof(float) * (size_t)n * n);
  /* Expand S once (the reference mirrors it tile by tile into its B cache). */
#pragma omp parallel for schedule(static)
  for (long k = 0; k < n; ++k)
    for (long j = 0; j < n; ++j) srow[(size_t)k * n + j] = sym_at(Sp, k, j, n);
#pragma omp parallel for schedule(static)
  for (long i = 0; i < M; ++i) {
    float* w = W + (size_t)i * n;
    for (long j = 0; j < n; ++j) w[j] = 0.0f;
    for (long k = 0; k < n; ++k) {
      const float a = A[(size_t)i * n + k];
      const float* s = srow + (size_t)k * n;
      for (long j = 0; j < n; ++j) w[j] = fmaf(a, s[j], w[j]);
    }
  }
  free(srow);
}

/* C = (A S) B: symmetric_matmul.cpp kernel, then gemm_benchmark.cpp kernel,
 * i.e. the two launches src/dsl/runner_cuda.py:147-197 run_graph makes. */
void orc_sandwich_f32(const float* A, const float* Sp, const float* B, float* C, int N) {
  float* W = (float*)malloc(sizeof(float) * (size_t)N * N);
  orc_symm_right_f32(A, Sp, W, N, N);
  orc_gemm_f32(W, B, C, N, N, N);
  free(W);
}

/* C(N x ncols) = T B with T[c][k] = g[N-1+k-c].  The reference computes only
 * X*T (toeplitz_matmul2.cpp:44-144); C = T*B is run through it as
 * (B^T T^T)^T with T^T's generator g[2N-2-k], keeping ascending k. */
void orc_toeplitz_left_f32(const float* g, const float* B, float* C, int N, int ncols) {
  const long n = N;
#pragma omp parallel for schedule(static)
  for (long c = 0; c < n; ++c) {
    float* out = C + (size_t)c * ncols;
    for (long r = 0; r < ncols; ++r) out[r] = 0.0f;
    for (long k = 0; k < n; ++k) {
      const float t = g[n - 1 + k - c];
      const float* b = B + (size_t)k * ncols;
      for (long r = 0; r < ncols; ++r) out[r] = fmaf(b[r], t, out[r]);
    }
  }
}

/* ---------------- elementwise sums and storage converters ---------------- */
/* Structure codes: 0 packed upper, 1 packed lower, 2 packed symmetric,
 * 3 diagonal, 4 Toeplitz generator (src/dsl/layout_functions.py:8-75). */
static inline size_t lidx(long i, long j) { return (size_t)(i * (i + 1) / 2 + j); }

static float struct_at(const float* S, int fmt, long n, long i, long j) {
  switch (fmt) {
    case 0: return i <= j ? S[pidx(i, j, n)] : 0.0f;                     /* upper_triangular_layout :8-23 */
    case 1: return j <= i ? S[lidx(i, j)] : 0.0f;                        /* lower_triangular_layout :25-36 */
    case 2: return i <= j ? S[pidx(i, j, n)] : S[pidx(j, i, n)];         /* symmetric_layout :50-68 */
    case 3: return i == j ? S[i] : 0.0f;                                 /* diagonal_layout :38-43 */
    default: return S[n - 1 + j - i];                                    /* toeplitz_layout :45-48 */
  }
}

/* C[k] = A[k] + B[k]: kernel_add_1d_vec4 (src/dsl/codegen_cuda.py:1745-1773),
 * one fp32 add per element in either of its branches. */
void orc_add_f32(const float* A, const float* B, float* C, long count) {
  for (long k = 0; k < count; ++k) C[k] = A[k] + B[k];
}

/* C = A + S expanded.  For the symmetric case this is kernel_add_gen_symm
 * (src/dsl/codegen_cuda.py:1665-1681): r = min(i,j), c = max(i,j),
 * C[i][j] = A[i][j] + S[r*n - r(r-1)/2 + (c-r)]. */
void orc_add_struct_f32(const float* A, const float* S, int fmt, float* C, int N) {
  const long n = N;
  for (long i = 0; i < n; ++i)
    for (long j = 0; j < n; ++j) C[i * n + j] = A[i * n + j] + struct_at(S, fmt, n, i, j);
}

/* D = the dense matrix of structured storage S. */
void orc_unpack_f32(const float* S, int fmt, float* D, int N) {
  const long n = N;
  for (long i = 0; i < n; ++i)
    for (long j = 0; j < n; ++j) D[i * n + j] = struct_at(S, fmt, n, i, j);
}

/* P = packed triangle of the dense D: upper (fmt 0 or 2) or lower (fmt 1). */
void orc_pack_f32(const float* D, int fmt, float* P, int N) {
  const long n = N;
  for (long i = 0; i < n; ++i)
    for (long j = 0; j < n; ++j) {
      if (fmt == 1 && j <= i) P[lidx(i, j)] = D[i * n + j];
      if (fmt != 1 && i <= j) P[pidx(i, j, n)] = D[i * n + j];
    }
}

/* g = generator of the rows x cols Toeplitz matrix T, as build_toeplitz_compact
 * (toeplitz_matmul2.cpp:34-41): g[rows-1-i] = T[i][0], g[rows-1+j] = T[0][j]. */
void orc_toeplitz_compact_f32(const float* T, float* g, int rows, int cols) {
  for (long i = 0; i < rows; ++i) g[rows - 1 - i] = T[i * cols];
  for (long j = 1; j < cols; ++j) g[rows - 1 + j] = T[j];
}

/* ---------------- fp64 ground truth on selected rows ---------------- */

/* out[r][:] = sum_k x_r[k] * B[k][:] in double, x_r given in double. */
static void rowvec_dense_f64(const double* x, const float* B, double* out, long K, long N) {
  for (long j = 0; j < N; ++j) out[j] = 0.0;
  for (long k = 0; k < K; ++k) {
    const double a = x[k];
    if (a == 0.0) continue;
    const float* b = B + (size_t)k * N;
    for (long j = 0; j < N; ++j) out[j] += a * (double)b[j];
  }
}

/* Rows `rows[0..nrows)` of A(MxK) B(KxN) in double, into out(nrows x N). */
void orc_gemm_rows_f64(const float* A, const float* B, const int* rows, int nrows, double* out, int N, int K) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    double* x = (double*)malloc(sizeof(double) * (size_t)K);
    for (long k = 0; k < K; ++k) x[k] = A[(size_t)rows[t] * K + k];
    rowvec_dense_f64(x, B, out + (size_t)t * N, K, N);
    free(x);
  }
}

/* Rows of U(packed upper) B(N x ncols) in double. */
void orc_upper_left_rows_f64(const float* Up, const float* B, const int* rows, int nrows, double* out, int N,
                             int ncols) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long c = rows[t];
    double* x = (double*)calloc((size_t)N, sizeof(double));
    for (long k = c; k < N; ++k) x[k] = Up[pidx(c, k, N)];
    rowvec_dense_f64(x, B, out + (size_t)t * ncols, N, ncols);
    free(x);
  }
}

/* Rows of T(from g) B(N x ncols) in double. */
void orc_toeplitz_left_rows_f64(const float* g, const float* B, const int* rows, int nrows, double* out, int N,
                                int ncols) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long c = rows[t];
    double* x = (double*)malloc(sizeof(double) * (size_t)N);
    for (long k = 0; k < N; ++k) x[k] = g[N - 1 + k - c];
    rowvec_dense_f64(x, B, out + (size_t)t * ncols, N, ncols);
    free(x);
  }
}

/* Rows of A S B (S packed symmetric) in double: w = A[i,:] S, then w B. */
void orc_sandwich_rows_f64(const float* A, const float* Sp, const float* B, const int* rows, int nrows,
                           double* out, int N) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long i = rows[t];
    double* w = (double*)calloc((size_t)N, sizeof(double));
    for (long k = 0; k < N; ++k) {
      const double a = A[(size_t)i * N + k];
      for (long j = 0; j < N; ++j) w[j] += a * (double)sym_at(Sp, k, j, N);
    }
    rowvec_dense_f64(w, B, out + (size_t)t * N, N, N);
    free(w);
  }
}

/* Rows of A S (S packed symmetric) in double. */
void orc_symm_right_rows_f64(const float* A, const float* Sp, const int* rows, int nrows, double* out, int M,
                             int N) {
  (void)M;
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long i = rows[t];
    double* w = out + (size_t)t * N;
    for (long j = 0; j < N; ++j) w[j] = 0.0;
    for (long k = 0; k < N; ++k) {
      const double a = A[(size_t)i * N + k];
      for (long j = 0; j < N; ++j) w[j] += a * (double)sym_at(Sp, k, j, N);
    }
  }
}

/* Normwise relative error ||X - R||_F / ||R||_F of fp32 rows X against fp64
 * rows R (n values each). */
double orc_relerr(const float* X, const double* R, size_t n) {
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const double d = (double)X[i] - R[i];
    num += d * d;
    den += R[i] * R[i];
  }
  return den > 0.0 ? sqrt(num / den) : sqrt(num);
}

/* ---------------- fp32 restatements on selected rows ----------------
 * Same FMA order as the full restatements above (and so as the reference
 * kernels), for checking the reference's own result at sizes where a full
 * CPU product is too slow. */

void orc_gemm_rows_f32(const float* A, const float* B, const int* rows, int nrows, float* out, int N, int K) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    float* c = out + (size_t)t * N;
    for (long j = 0; j < N; ++j) c[j] = 0.0f;
    for (long k = 0; k < K; ++k) {
      const float a = A[(size_t)rows[t] * K + k];
      const float* b = B + (size_t)k * N;
      for (long j = 0; j < N; ++j) c[j] = fmaf(a, b[j], c[j]);
    }
  }
}

void orc_upper_left_rows_f32(const float* Up, const float* B, const int* rows, int nrows, float* out, int N,
                             int ncols) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long c = rows[t];
    float* o = out + (size_t)t * ncols;
    for (long r = 0; r < ncols; ++r) o[r] = 0.0f;
    for (long k = N - 1; k >= c; --k) {
      const float u = Up[pidx(c, k, N)];
      const float* b = B + (size_t)k * ncols;
      for (long r = 0; r < ncols; ++r) o[r] = fmaf(b[r], u, o[r]);
    }
  }
}

void orc_toeplitz_left_rows_f32(const float* g, const float* B, const int* rows, int nrows, float* out, int N,
                                int ncols) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long c = rows[t];
    float* o = out + (size_t)t * ncols;
    for (long r = 0; r < ncols; ++r) o[r] = 0.0f;
    for (long k = 0; k < N; ++k) {
      const float v = g[N - 1 + k - c];
      const float* b = B + (size_t)k * ncols;
      for (long r = 0; r < ncols; ++r) o[r] = fmaf(b[r], v, o[r]);
    }
  }
}

void orc_sandwich_rows_f32(const float* A, const float* Sp, const float* B, const int* rows, int nrows, float* out,
                           int N) {
#pragma omp parallel for schedule(dynamic, 1)
  for (long t = 0; t < nrows; ++t) {
    const long i = rows[t];
    float* w = (float*)calloc((size_t)N, sizeof(float));
    for (long k = 0; k < N; ++k) {
      const float a = A[(size_t)i * N + k];
      for (long j = 0; j < N; ++j) w[j] = fmaf(a, sym_at(Sp, k, j, N), w[j]);
    }
    float* c = out + (size_t)t * N;
    for (long j = 0; j < N; ++j) c[j] = 0.0f;
    for (long k = 0; k < N; ++k) {
      const float a = w[k];
      const float* b = B + (size_t)k * N;
      for (long j = 0; j < N; ++j) c[j] = fmaf(a, b[j], c[j]);
    }
    free(w);
  }
}
