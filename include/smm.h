/* smm.h — C ABI of libsmm, the B200 (sm_100a) structured matrix-multiply library.
 *
 * Plain pointers and sizes only.  Every matrix is row-major fp32 in device
 * memory owned by the caller; the library never allocates user outputs.
 * Every entry point returns an smm_status and never exits the process; the
 * thread-local text of the last failure is available from smm_last_error().
 * Calls are asynchronous on the given stream (NULL = the legacy default
 * stream) unless stated otherwise.
 *
 * Storage conventions, as defined by the reference DSL
 * (src/dsl/layout_functions.py) and its CUDA runner (src/dsl/runner_cuda.py):
 *   packed upper / symmetric  row-major upper triangle incl. diagonal,
 *                             idx(i,j) = i*N - i*(i-1)/2 + (j-i) for i <= j,
 *                             N*(N+1)/2 floats (layout_functions.py:8-23,
 *                             50-68; runner_cuda.py:96-97)
 *   diagonal                  N floats (layout_functions.py:38-43;
 *                             runner_cuda.py:98-99)
 *   Toeplitz                  2N-1 generator, T[i][j] = g[(N-1) + (j-i)]
 *                             (layout_functions.py:45-48; Cuda
 *                             kernels/toeplitz.cu:91, 255-262)
 *
 * Arithmetic modes of the tensor-core contractions:
 *   SMM_MODE_3XTF32  fp32 semantics: each operand x = hi + lo with
 *                    hi = tf32(x), lo = x - hi; C = hi*hi + hi*lo + lo*hi,
 *                    fp32 accumulation in tensor memory (3 MMA passes)
 *   SMM_MODE_TF32    one TF32 pass (fast, ~1e-3 relative)
 *   SMM_MODE_BF16    operands rounded to bf16 (inside the call), fp32
 *                    accumulation
 *
 * A packed upper / symmetric / lower operand of an entry point with a
 * workspace is expanded into a dense copy there (fp32, or bf16 in bf16 mode)
 * and read by TMA; the *_workspace_size functions include that copy.  Given
 * less workspace (at least the rest of the requirement) the entry point builds
 * the operand on chip from its packed rows instead (slower), so callers that
 * sized the workspace without the copy keep working.  Both give results
 * within the mode's tolerance; SMM_EXPAND=0 in the environment forces the
 * on-chip path.
 */
#ifndef SMM_H
#define SMM_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SMM_OK = 0,
  SMM_ERR_INVALID = 1,        /* bad pointer, shape, mode or format */
  SMM_ERR_CUDA = 2,           /* a CUDA runtime/driver call failed */
  SMM_ERR_NCCL = 3,           /* reserved for the multi-GPU layer */
  SMM_ERR_DEVICE_TIMEOUT = 4, /* a kernel's bounded wait expired; the kernel exited cleanly */
  SMM_ERR_WORKSPACE = 5,      /* caller workspace missing or too small */
  SMM_ERR_UNSUPPORTED = 6,    /* device is not sm_100 or feature not built */
  SMM_ERR_BOUNDS = 7          /* bounds-checked debug build (libsmm_debug.so): an out-of-range read was
                                 caught and skipped */
} smm_status;

typedef enum { SMM_MODE_3XTF32 = 0, SMM_MODE_TF32 = 1, SMM_MODE_BF16 = 2 } smm_mode;
typedef enum { SMM_FMT_PACKED = 0, SMM_FMT_DENSE = 1 } smm_format;
/* Structured storage formats of the elementwise and converter entry points:
 * packed upper, packed lower (row-major lower triangle incl. diagonal,
 * idx(i,j) = i*(i+1)/2 + j for j <= i, layout_functions.py:25-36), packed
 * symmetric (upper storage, mirrored), diagonal (N floats), Toeplitz (2N-1
 * generator). */
typedef enum {
  SMM_STRUCT_UPPER = 0,
  SMM_STRUCT_LOWER = 1,
  SMM_STRUCT_SYMM = 2,
  SMM_STRUCT_DIAG = 3,
  SMM_STRUCT_TOEPLITZ = 4
} smm_struct;

/* ---- library ---------------------------------------------------------- */

/* Thread-local message describing the last non-OK status ("" if none). */
const char* smm_last_error(void);
/* Library version as 10000*major + 100*minor + patch. */
int smm_version(void);
/* Number of kernel launches this library has issued in this process. */
unsigned long long smm_launch_count(void);
/* Synchronises `stream`, then reads and clears this device's sticky kernel
 * status word: SMM_ERR_DEVICE_TIMEOUT if any kernel since the last call gave
 * up a bounded wait (it then wrote no output and exited cleanly), else SMM_OK. */
int smm_device_status(void* stream);

/* ---- diagonal scaling (HBM-bound, no tensor cores, bit-exact) ---------- */

/* C[i][j] = d[i] * B[i][j], B and C M x N (ldb = ldc = N).  One fp32 multiply
 * per element, no contraction.  Replaces kernel_diag_x_gen + its wrapper
 * (src/dsl/codegen_cuda.py:1253-1332), the DSL's DiagonalMatrix @
 * GeneralMatrix. */
int smm_diag_rows(const float* d, const float* B, float* C, int M, int N, void* stream);

/* C[i][j] = A[i][j] * b[j] (column scale).  Replaces kernel_gen_x_diag
 * (src/dsl/codegen_cuda.py:808-964) and gemm_diag (Cuda kernels/diagonal.cu:44-148). */
int smm_diag_cols(const float* A, const float* b, float* C, int M, int N, void* stream);

/* Row scale with HOST (ideally pinned) buffers: copies d and B in, scales and
 * copies C out in row chunks on two internal streams so the transfers in
 * both directions overlap each other and the kernel.  Synchronous.  dev_ws
 * must hold smm_diag_rows_host_workspace_size(M, N) bytes of device memory. */
size_t smm_diag_rows_host_workspace_size(int M, int N);
int smm_diag_rows_host(const float* d_host, const float* B_host, float* C_host, int M, int N, void* dev_ws,
                       size_t ws_bytes);

/* ---- tensor-core contractions (tcgen05 + TMEM, TMA-fed) ---------------- */

/* Workspace (device bytes) an entry point needs for the given shape/mode;
 * 0 means none.  Passing a larger workspace is always allowed. */
size_t smm_gemm_workspace_size(int M, int N, int K, int mode);
size_t smm_upper_left_workspace_size(int N, int ncols, int u_fmt, int mode);
size_t smm_toeplitz_left_workspace_size(int N, int ncols, int mode);
size_t smm_symm_sandwich_workspace_size(int N, int mode);
size_t smm_symm_left_workspace_size(int N, int ncols, int mode);

/* C(MxN) = A(MxK) B(KxN).  Replaces kernel_gen_x_gen + wrapper
 * (src/dsl/codegen_cuda.py:62-278) and KernelOptimized::run
 * (Cuda kernels/gemmoptimized.cu:249-272). */
int smm_gemm(const float* A, const float* B, float* C, int M, int N, int K, int mode, void* ws, size_t ws_bytes,
             void* stream);

/* C(N x ncols) = U(NxN upper) B(N x ncols).  u_fmt SMM_FMT_PACKED: U packed
 * upper (N(N+1)/2 floats); SMM_FMT_DENSE: U a dense N x N array whose strict
 * lower part is exactly zero (never read).  All-zero tiles of U are skipped;
 * only diagonal tiles are masked.  Left-side counterpart of kernel_gen_x_upper
 * (src/dsl/codegen_cuda.py:280-544) and Cuda kernels/upper.cu:177-313, which
 * compute A*U. */
int smm_upper_left(const float* U, int u_fmt, const float* B, float* C, int N, int ncols, int mode, void* ws,
                   size_t ws_bytes, void* stream);

/* C(N x ncols) = T B, T the N x N Toeplitz matrix of generator g[2N-1].  The
 * generator is expanded on chip; HBM traffic is B and C only.  Left-side
 * counterpart of gemm_toeplitz_double_buffer (Cuda kernels/toeplitz.cu:158-253),
 * which computes A*T; the DSL has no CUDA lowering for ToeplitzMatrix
 * (src/dsl/codegen_cuda.py:1681-1682). */
int smm_toeplitz_left(const float* g, const float* B, float* C, int N, int ncols, int mode, void* ws,
                      size_t ws_bytes, void* stream);

/* C(N x ncols) = S B, S symmetric given packed upper (expanded into a dense
 * copy in the workspace, or mirrored on chip without room for it).
 * Replaces kernel_symm_x_gen (src/dsl/codegen_cuda.py:973-1245). */
int smm_symm_left(const float* S_packed, const float* B, float* C, int N, int ncols, int mode, void* ws,
                  size_t ws_bytes, void* stream);

/* Row slabs of the three structured products, for partitioning a product
 * by output rows (one slab per GPU): C (nrows x ncols) = X[row0 : row0+nrows, :] B,
 * X being the N x N upper-triangular / Toeplitz / symmetric operand.  The
 * full-matrix entry points above are the slab [0, N).  For the triangular
 * operand a slab's K range starts at row0 (zero tiles are never visited). */
int smm_upper_left_rows(const float* U, int u_fmt, const float* B, float* C, int N, int ncols, int row0, int nrows,
                        int mode, void* ws, size_t ws_bytes, void* stream);
int smm_toeplitz_left_rows(const float* g, const float* B, float* C, int N, int ncols, int row0, int nrows,
                           int mode, void* ws, size_t ws_bytes, void* stream);
int smm_symm_left_rows(const float* S_packed, const float* B, float* C, int N, int ncols, int row0, int nrows,
                       int mode, void* ws, size_t ws_bytes, void* stream);

/* C = A S B (all N x N, S packed upper symmetric), computed as A (S B) with
 * the intermediate in the workspace.  Replaces the two launches
 * src/dsl/runner_cuda.py:147-197 run_graph makes for A@S@B
 * (kernel_gen_x_symm, src/dsl/codegen_cuda.py:546-806, then kernel_gen_x_gen). */
int smm_symm_sandwich(const float* A, const float* S_packed, const float* B, float* C, int N, int mode, void* ws,
                      size_t ws_bytes, void* stream);

/* Allocation-free variant of smm_symm_sandwich (no counterpart in the
 * reference).  For callers that cannot allocate device memory: code inside a
 * host framework that owns all device memory through its own pool, or a
 * latency-critical path where cudaMalloc's implicit device synchronisation is
 * not acceptable.  The S*B intermediate (and padded copies of A and B when
 * N % 4 != 0 or they are not 16-byte aligned) lives in a fixed 16 MiB static
 * device array inside libsmm, which every GPU that loads the library holds
 * until process exit: N <= 2048 in the fp32 modes with N % 4 == 0 and
 * 16-byte-aligned A, B, N <= 1180 when padded copies are needed, N <= 1294
 * in bf16 mode (the bf16 copies share it).  S is expanded into a dense copy
 * only when the scratch has room left for it (fp32 aligned: N <= 1448), else
 * mirrored on chip.  Larger N returns SMM_ERR_WORKSPACE.  Calls no
 * cudaMalloc/cudaFree.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and must come before any stream
 * capture.  Every call shares the one array and it keeps the last call's
 * contents: calls that overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller. */
int smm_symm_sandwich_noalloc(const float* A, const float* S_packed, const float* B, float* C, int N, int mode,
                              void* stream);

/* ---- multi-GPU products (one process per GPU, NCCL over NVLink) ------- */

/* A product C = X B is partitioned by output row slabs, one per rank (GPU).
 * The shared right operand B reaches every rank inside each call, in column
 * blocks, on the communicator's high-priority stream, and this rank computes
 * the block's columns of its slab as soon as the block has landed, on
 * internal compute streams joined back into `stream` before the call's work
 * ends, so the transfer of later blocks overlaps the tensor-core work on
 * earlier ones.  B comes either from one root rank (`root` = its rank; the
 * root packs each block contiguously and broadcasts it; B is read on the
 * root only, the other ranks may pass NULL), or sharded by rows (`root` =
 * SMM_MG_SHARDED: each rank passes its share, rows [rank * s, min(K, (rank +
 * 1) * s)) of B with s = smm_mg_share_rows(K, world), and the blocks are
 * all-gathered from the shares).  Either way B's rows are 16-byte aligned.
 * In bf16 mode the blocks travel as bf16 (half the bytes; the same rounding
 * as the single-GPU conversion).  Every output element comes from one
 * full-K contraction: the slab equals the single-GPU entry point's rows.
 * Calls are collective: every rank makes the same calls with the same
 * shapes, mode and root, in the same order.  No kernel reads another GPU's
 * memory.  The reference has no multi-GPU code; this is the row-slab
 * partition with the shared operand sent over NVLink that its single-GPU
 * kernels scale to.  NCCL is loaded at run time (libnccl.so.2, the copy
 * already in the process when there is one).  At world = 1 the calls
 * compute without any collective. */
#define SMM_MG_SHARDED (-1)
/* `root` = SMM_MG_REPLICATED: B is whole on every rank (and the sandwich's S):
 * nothing travels, every rank computes its rows from its own B in place. */
#define SMM_MG_REPLICATED (-2)
#define SMM_MG_ID_BYTES 128
typedef struct smm_mg_comm smm_mg_comm;

/* NCCL unique id (SMM_MG_ID_BYTES bytes) made on one rank and handed to the
 * others by any host means before smm_mg_comm_init. */
int smm_mg_unique_id(void* id_out);
/* Communicator of rank `rank` of `world` on the current device (collective:
 * blocks until every rank has joined). */
int smm_mg_comm_init(smm_mg_comm** comm, int rank, int world, const void* id);
/* Waits for this rank's collectives and compute streams, then frees the
 * communicator. */
int smm_mg_comm_destroy(smm_mg_comm* comm);
/* Frees the communicator without waiting for peers (a failed or departed
 * rank): pending collectives end with an error instead of blocking. */
int smm_mg_comm_abort(smm_mg_comm* comm);
/* SMM_ERR_NCCL if the communicator saw an asynchronous NCCL error. */
int smm_mg_comm_status(smm_mg_comm* comm);

/* Row-slab boundaries bounds[0] = 0 <= ... <= bounds[world] = N on 256-row
 * tiles (a CTA-pair tile's height), minimising the largest slab's work: rows
 * cost 1, or N - i for an upper-triangular left operand (triangular != 0). */
int smm_mg_row_slabs(int N, int world, int triangular, int* bounds);
/* Column-block boundaries the calls use for a transfer of B's ncols columns
 * at this world size (bounds needs 17 ints); returns the block count: 1 at
 * world 1, 4 at world 2, 2 at 3-4, 1 from 5 up (SMM_MG_CHUNKS in the
 * environment sets it, 1 .. 16). */
int smm_mg_chunks(int ncols, int world, int* bounds);
/* The same for a copy-engine gather of a sharded B (smm_mg_enable_copy_engines),
 * whose pushes take no SM: 4 blocks at every world size above 1
 * (SMM_MG_CHUNKS sets it, 1 .. 16).  No counterpart in the reference (it has
 * no multi-GPU code). */
int smm_mg_gather_chunks(int ncols, int world, int* bounds);

/* Copy-engine gather of a sharded B (collective; at most 8 ranks on one
 * node).  Every rank allocates plane_bytes of device memory (the same count
 * on every rank) and maps every peer's allocation through CUDA IPC; from
 * then on a sharded call whose column blocks fit (smm_mg_plane_bytes) packs
 * this rank's share of each block into its slot of its own buffer and the
 * copy engines push that slot into every peer's buffer -- no NCCL kernel and
 * no SM in the transfer, which therefore runs beside the contractions.
 * Interprocess events order the pushes against the consumers, and two host
 * barriers per call (POSIX shared memory named by the unique id) order the
 * event records across processes.  Enabling again replaces the buffer;
 * smm_mg_comm_destroy releases it. */
size_t smm_mg_plane_bytes(const smm_mg_comm* comm, int K, int ncols, int mode);
int smm_mg_enable_copy_engines(smm_mg_comm* comm, size_t plane_bytes);
int smm_mg_copy_engines_enabled(const smm_mg_comm* comm);

/* Rows in each rank's share of a K-row B sharded over `world` ranks:
 * ceil(K / world) (the last shares may hold fewer rows of B, or none). */
int smm_mg_share_rows(int K, int world);

/* C_slab (nrows x N) = A_slab (nrows x K, this rank's rows of A) B (K x N). */
size_t smm_mg_gemm_workspace_size(const smm_mg_comm* comm, int nrows, int N, int K, int mode);
int smm_mg_gemm(smm_mg_comm* comm, const float* A_slab, const float* B, float* C_slab, int nrows, int N, int K,
                int mode, int root, void* ws, size_t ws_bytes, void* stream);
/* C_slab (nrows x ncols) = U[row0 : row0+nrows, :] B, U packed upper (the whole
 * packed array on every rank; only the slab's rows are read). */
size_t smm_mg_upper_left_workspace_size(const smm_mg_comm* comm, int N, int ncols, int nrows, int mode);
int smm_mg_upper_left(smm_mg_comm* comm, const float* U_packed, const float* B, float* C_slab, int N, int ncols,
                      int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes, void* stream);
/* Interleaved ownership of U's rows (the alternative to one contiguous slab
 * per rank): U's 256-row tiles in decreasing order of work each go to the
 * rank with the least work so far, so every rank holds long and short rows
 * alike and the ranks' tile schedules come out even (32 tiles on 8 ranks:
 * {r, 15 - r, 16 + r, 31 - r}).  Writes this rank's tile indices, ascending,
 * into tiles (room for max_tiles; ceil(N / 256) always suffices) and their
 * number into *count.  No counterpart in the reference (it has no
 * multi-GPU code). */
int smm_mg_upper_row_tiles(int N, int world, int rank, int* tiles, int max_tiles, int* count);
/* C_rows = the rows of U B in this rank's row tiles (ascending indices of
 * 256-row tiles of U, at most 64), stacked in that order: tile i's rows at
 * C_rows + (256 i) ncols (the last tile of U may be shorter).  U packed upper
 * on every rank; B as for the other calls.  One call moves B once and
 * computes all the tiles.  No counterpart in the reference. */
size_t smm_mg_upper_left_tiles_workspace_size(const smm_mg_comm* comm, int N, int ncols, int ntiles, int mode);
int smm_mg_upper_left_tiles(smm_mg_comm* comm, const float* U_packed, const float* B, float* C_rows, int N,
                            int ncols, const int* tiles, int ntiles, int mode, int root, void* ws, size_t ws_bytes,
                            void* stream);
/* C_slab (nrows x ncols) = T[row0 : row0+nrows, :] B, T of generator g[2N-1]
 * (on every rank). */
size_t smm_mg_toeplitz_left_workspace_size(const smm_mg_comm* comm, int N, int ncols, int mode);
int smm_mg_toeplitz_left(smm_mg_comm* comm, const float* g, const float* B, float* C_slab, int N, int ncols,
                         int row0, int nrows, int mode, int root, void* ws, size_t ws_bytes, void* stream);
/* C_slab (nrows x N) = (A_slab S) B, S packed symmetric (the root's input,
 * rank 0's when B is sharded; a receive buffer of N(N+1)/2 floats on the
 * other ranks): the reference's run_graph order, (A S) then times B, per row
 * slab. */
size_t smm_mg_symm_sandwich_workspace_size(const smm_mg_comm* comm, int N, int nrows, int mode);
int smm_mg_symm_sandwich(smm_mg_comm* comm, const float* A_slab, float* S_packed, const float* B, float* C_slab,
                         int N, int nrows, int mode, int root, void* ws, size_t ws_bytes, void* stream);

/* ---- host-buffer contractions ------------------------------------------ */

/* The contractions above with A, B, C (and U, S, g) in HOST memory: the
 * drop-in for callers of the reference's CPU kernels, which take host arrays
 * (Cuda kernels/gemm_benchmark.cpp:40-156 compute_matrix_multi1,
 * upper_triag_matmul.cpp:41-137, symmetric_matmul.cpp:84-211,
 * toeplitz_matmul2.cpp:44-144).  Pinned host buffers let the copies overlap:
 * the left operand(s) cross PCIe once and are prepared on the device (a
 * packed operand expanded), then B streams through in column chunks on two
 * internal streams, each chunk's copy-in, product and copy-out overlapping
 * the neighbouring chunks'.  Synchronous; results equal the device entry
 * points' within the mode's tolerance.  dev_ws must hold the matching
 * *_host_workspace_size bytes of device memory (16-byte aligned), with no
 * pending work on it: the calls run on internal streams that are not
 * ordered after the caller's streams.  Host threads may call them
 * concurrently, each with its own workspace; calls on one device share its
 * two internal streams (created on the first call) and so run one after
 * another on the GPU. */
size_t smm_gemm_host_workspace_size(int M, int N, int K, int mode);
int smm_gemm_host(const float* A, const float* B, float* C, int M, int N, int K, int mode, void* dev_ws,
                  size_t ws_bytes);
size_t smm_upper_left_host_workspace_size(int N, int ncols, int mode);
int smm_upper_left_host(const float* U_packed, const float* B, float* C, int N, int ncols, int mode, void* dev_ws,
                        size_t ws_bytes);
size_t smm_symm_left_host_workspace_size(int N, int ncols, int mode);
int smm_symm_left_host(const float* S_packed, const float* B, float* C, int N, int ncols, int mode, void* dev_ws,
                       size_t ws_bytes);
size_t smm_toeplitz_left_host_workspace_size(int N, int ncols, int mode);
int smm_toeplitz_left_host(const float* g, const float* B, float* C, int N, int ncols, int mode, void* dev_ws,
                           size_t ws_bytes);
size_t smm_symm_sandwich_host_workspace_size(int N, int mode);
int smm_symm_sandwich_host(const float* A, const float* S_packed, const float* B, float* C, int N, int mode,
                           void* dev_ws, size_t ws_bytes);

/* The reference CPU drivers' own orientation with HOST arrays: C (M x N) =
 * A (M x K) X, X packed upper (upper_triag_matmul.cpp:41-137), packed
 * symmetric (symmetric_matmul.cpp:84-211) or a Toeplitz generator of K+N-1
 * floats (toeplitz_matmul2.cpp:44-144); K = N for the packed ones.  X crosses
 * PCIe once and is expanded on the device; A goes through in row chunks on
 * two internal streams, each chunk's copy-in, product and copy-out
 * overlapping the neighbouring chunks'.  Synchronous; workspace and stream
 * rules as for the host-buffer entries above. */
size_t smm_gen_x_upper_host_workspace_size(int M, int N, int mode);
int smm_gen_x_upper_host(const float* A, const float* U_packed, float* C, int M, int N, int mode, void* dev_ws,
                         size_t ws_bytes);
size_t smm_gen_x_symm_host_workspace_size(int M, int N, int mode);
int smm_gen_x_symm_host(const float* A, const float* S_packed, float* C, int M, int N, int mode, void* dev_ws,
                        size_t ws_bytes);
size_t smm_gen_x_toeplitz_host_workspace_size(int M, int N, int K, int mode);
int smm_gen_x_toeplitz_host(const float* A, const float* g, float* C, int M, int N, int K, int mode, void* dev_ws,
                            size_t ws_bytes);

/* Column scale with HOST buffers, C = A diag(b) (diag_matmul.cpp:45-111
 * optimized_compute, the reference driver's orientation): b is copied once,
 * A and C go through in row chunks on two internal streams.  Synchronous,
 * bit-exact; dev_ws must hold smm_diag_cols_host_workspace_size(M, N) bytes. */
size_t smm_diag_cols_host_workspace_size(int M, int N);
int smm_diag_cols_host(const float* A_host, const float* b_host, float* C_host, int M, int N, void* dev_ws,
                       size_t ws_bytes);

/* ---- structured right operand (the reference's own orientation) ------- */

/* Workspace for smm_gen_x_upper / smm_gen_x_symm / smm_gen_x_lower: a padded
 * (or bf16) copy of A, plus the dense expansion of the packed right operand
 * (see the note on packed operands above; without room for it the operand is
 * built on chip by the transform warps). */
size_t smm_gen_x_struct_workspace_size(int M, int N, int mode);

/* C(M x N) = A(M x N) U(N x N, packed upper).  Replaces kernel_gen_x_upper +
 * copy_B_to_Reg_Upper (src/dsl/codegen_cuda.py:280-544) and Cuda
 * kernels/upper.cu:73-313.  K-blocks below a column tile's diagonal are
 * never visited. */
int smm_gen_x_upper(const float* A, const float* U_packed, float* C, int M, int N, int mode, void* ws,
                    size_t ws_bytes, void* stream);

/* C(M x N) = A(M x N) S(N x N, packed upper symmetric).
 * Replaces kernel_gen_x_symm + copy_B_to_Reg_Symm (src/dsl/codegen_cuda.py:546-806)
 * and Cuda kernels/symmetric.cu:76-271. */
int smm_gen_x_symm(const float* A, const float* S_packed, float* C, int M, int N, int mode, void* ws,
                   size_t ws_bytes, void* stream);

/* C(M x N) = A(M x N) L(N x N, packed lower, idx(i,j) = i(i+1)/2 + j).
 * Replaces the DSL's GeneralMatrix @ LowerTriangularMatrix, which the
 * reference implements only in its CPU AVX backend
 * (src/dsl/codegen_multiply_avx.py:546-642).  K-blocks above a column tile's
 * diagonal are never visited.  Workspace: smm_gen_x_struct_workspace_size. */
int smm_gen_x_lower(const float* A, const float* L_packed, float* C, int M, int N, int mode, void* ws,
                    size_t ws_bytes, void* stream);

/* C(M x N) = A(M x K) T(K x N), T the Toeplitz matrix of generator
 * g[K+N-1], T[k][n] = g[(K-1) + (n-k)]: the orientation of the reference's
 * Toeplitz kernels, gemm_toeplitz_double_buffer (Cuda kernels/toeplitz.cu:
 * 76-253, t_idx = (K-1)+(n-k) at :91) and compute_matrix_multi1
 * (toeplitz_matmul2.cpp:44-144).  With smm_gen_x_toeplitz_workspace_size
 * bytes T is expanded into a dense copy and read by TMA; with room for the
 * staged A only, T is built on chip from the generator. */
size_t smm_gen_x_toeplitz_workspace_size(int M, int N, int K, int mode);
int smm_gen_x_toeplitz(const float* A, const float* g, float* C, int M, int N, int K, int mode, void* ws,
                       size_t ws_bytes, void* stream);

/* C(N x N) = S1 S2, both packed upper symmetric.  Replaces kernel_symm_x_symm
 * (src/dsl/codegen_cuda.py:1340-1613).  No workspace: both operands are built
 * on chip from their packed rows. */
int smm_symm_x_symm(const float* S1_packed, const float* S2_packed, float* C, int N, int mode, void* stream);

/* The same product with a workspace: given smm_symm_x_symm_workspace_size
 * bytes, both operands are expanded into dense copies there and read by TMA
 * (about 2.5x faster at N = 8192); given less, as smm_symm_x_symm. */
size_t smm_symm_x_symm_workspace_size(int N, int mode);
int smm_symm_x_symm_ws(const float* S1_packed, const float* S2_packed, float* C, int N, int mode, void* ws,
                       size_t ws_bytes, void* stream);

/* ---- lower-triangular operands (packed lower, idx(i,j) = i(i+1)/2 + j) ---- */

size_t smm_lower_left_workspace_size(int N, int ncols, int mode);

/* C(N x ncols) = L B, L packed lower.  The left-side counterpart of
 * smm_upper_left (the DSL's LowerTriangularMatrix @ GeneralMatrix; the
 * reference's lower-triangular layout is src/dsl/layout_functions.py:25-36).
 * K-blocks right of a row tile's diagonal are never visited. */
int smm_lower_left(const float* L_packed, const float* B, float* C, int N, int ncols, int mode, void* ws,
                   size_t ws_bytes, void* stream);

/* C(N x N) = L1 L2, both packed lower.  Replaces the DSL's
 * LowerTriangularMatrix @ LowerTriangularMatrix of the reference's CPU AVX
 * backend (src/dsl/codegen_multiply_avx.py:644-923).  Output tiles wholly
 * above the diagonal are written as zeros without a K loop.  No workspace. */
int smm_lower_x_lower(const float* L1_packed, const float* L2_packed, float* C, int N, int mode, void* stream);

/* The same product with a workspace: given smm_lower_x_lower_workspace_size
 * bytes, both operands are expanded into dense copies there and read by TMA,
 * with the same K-range clipping; given less, as smm_lower_x_lower. */
size_t smm_lower_x_lower_workspace_size(int N, int mode);
int smm_lower_x_lower_ws(const float* L1_packed, const float* L2_packed, float* C, int N, int mode, void* ws,
                         size_t ws_bytes, void* stream);

/* ---- elementwise sums and storage converters (HBM-bound, bit-exact) ---- */

/* C[k] = A[k] + B[k] for k < count: the DSL's `+` of two operands in the same
 * storage (general + general over M*N floats, symmetric/upper/lower + the
 * same class over N(N+1)/2, diagonal + diagonal over N).  One IEEE fp32 add
 * per element.  Replaces kernel_add_1d_vec4 + wrapper
 * (src/dsl/codegen_cuda.py:1718-1812). */
int smm_add(const float* A, const float* B, float* C, long long count, void* stream);

/* C = A + S, A and C dense N x N, S in structured storage s_fmt (an
 * smm_struct) expanded on the fly: C[i][j] = A[i][j] + S(i,j).  For
 * SMM_STRUCT_SYMM this replaces kernel_add_gen_symm + wrapper
 * (src/dsl/codegen_cuda.py:1650-1716), the DSL's GeneralMatrix +
 * SymmetricMatrix. */
int smm_add_struct(const float* A, const float* S, int s_fmt, float* C, int N, void* stream);

/* D (dense N x N) = the structured matrix S (s_fmt): zeros outside the
 * triangle / diagonal, the mirror for SMM_STRUCT_SYMM, T[i][j] =
 * g[N-1+j-i] for SMM_STRUCT_TOEPLITZ (layout_functions.py:8-75). */
int smm_unpack(const float* S, int s_fmt, float* D, int N, void* stream);

/* P (packed, N(N+1)/2 floats) = the upper (SMM_STRUCT_UPPER or _SYMM) or
 * lower (SMM_STRUCT_LOWER) triangle of the dense N x N matrix D, in the DSL's
 * packed order (layout_functions.py:8-36; the torch.triu_indices order of
 * main2.py:44-45 and runner_cuda.py:96-97). */
int smm_pack(const float* D, int s_fmt, float* P, int N, void* stream);

/* g (rows + cols - 1 floats) = the generator of the rows x cols Toeplitz
 * matrix T: g[rows-1-i] = T[i][0], g[rows-1+j] = T[0][j].  Replaces
 * build_toeplitz_compact (Cuda kernels/toeplitz.cu:254-261,
 * toeplitz_matmul2.cpp:34-41). */
int smm_toeplitz_compact(const float* T, float* g, int rows, int cols, void* stream);

/* ---- reference-compatible wrappers (synchronous, timed) ---------------- */

/* One per operation the DSL's CUDA runner generates, with the generated
 * wrapper's calling convention <Out>_computation(lhs_data, rhs_data,
 * out_data, gflops_out, n, time_ms_out) (src/dsl/codegen_cuda.py:44-45,
 * 250-275): device pointers in the DSL's storage formats, a square order n,
 * synchronous on the legacy default stream, the kernels timed with CUDA
 * events into *time_ms_out, and *gflops_out counted as the generated wrappers
 * do (2 n^3 for a product; n^2 for a diagonal scale or a sum).  fp32
 * (3xTF32) mode.  Any workspace is allocated stream-ordered outside the timed
 * window.  Returns a status (the generated wrappers ignore errors; a ctypes
 * caller that sets no restype may do the same).  Each replaces the generated
 * wrapper of the kernel named: */
int smm_compat_gen_x_gen(const float* A, const float* B, float* C, float* gflops_out, int n, float* time_ms_out);      /* kernel_gen_x_gen :62-278 */
int smm_compat_diag_x_gen(const float* d, const float* B, float* C, float* gflops_out, int n, float* time_ms_out);     /* kernel_diag_x_gen :1253-1332 */
int smm_compat_gen_x_diag(const float* A, const float* d, float* C, float* gflops_out, int n, float* time_ms_out);     /* kernel_gen_x_diag :808-964 */
int smm_compat_upper_x_gen(const float* U, const float* B, float* C, float* gflops_out, int n, float* time_ms_out);    /* no CUDA kernel in the reference (:1681) */
int smm_compat_toeplitz_x_gen(const float* g, const float* B, float* C, float* gflops_out, int n, float* time_ms_out); /* no CUDA kernel in the reference (:1681) */
int smm_compat_symm_x_gen(const float* S, const float* B, float* C, float* gflops_out, int n, float* time_ms_out);     /* kernel_symm_x_gen :973-1245 */
int smm_compat_gen_x_symm(const float* A, const float* S, float* C, float* gflops_out, int n, float* time_ms_out);     /* kernel_gen_x_symm :546-806 */
int smm_compat_gen_x_upper(const float* A, const float* U, float* C, float* gflops_out, int n, float* time_ms_out);    /* kernel_gen_x_upper :280-544 */
int smm_compat_symm_x_symm(const float* S1, const float* S2, float* C, float* gflops_out, int n, float* time_ms_out);  /* kernel_symm_x_symm :1340-1613 */
int smm_compat_gen_x_lower(const float* A, const float* L, float* C, float* gflops_out, int n, float* time_ms_out);    /* CPU AVX backend only */
int smm_compat_lower_x_gen(const float* L, const float* B, float* C, float* gflops_out, int n, float* time_ms_out);    /* none in the reference */
int smm_compat_lower_x_lower(const float* L1, const float* L2, float* C, float* gflops_out, int n, float* time_ms_out);/* CPU AVX backend only */
int smm_compat_add_gen_symm(const float* A, const float* S, float* C, float* gflops_out, int n, float* time_ms_out);   /* kernel_add_gen_symm :1650-1716 */
/* A S B in one call: run_graph's two generated launches (src/dsl/runner_cuda.py:147-197). */
int smm_compat_symm_sandwich(const float* A, const float* S, const float* B, float* C, float* gflops_out, int n,
                             float* time_ms_out);

/* ---- failure-detection probe ------------------------------------------- */

/* Launches one CTA that waits on a shared-memory barrier nothing ever
 * arrives on, with the given wait limit (ns), exactly like the pipeline
 * waits in the contraction kernels.  Returns SMM_ERR_DEVICE_TIMEOUT when the
 * limit expired and the kernel exited cleanly (the expected outcome); used
 * to test the timeout path without faulting or hanging the GPU. */
int smm_debug_timeout_probe(unsigned long long wait_limit_ns, void* stream);

/* Diagnostic: the next tensor-core contraction launched from the calling
 * thread records the state of its first CTA into `trace` (64 device words:
 * tensor-memory base, k-block count, first staged operand words, matrix and
 * instruction descriptors, first accumulator words).  NULL disables. */
int smm_debug_trace_next(unsigned* trace);

/* Measurement: the next tensor-core contraction kernel launched from the
 * calling thread is bracketed by cudaEventRecord(event_before) and
 * cudaEventRecord(event_after) (cudaEvent_t handles) on its stream, so that
 * kernel can be timed alone, without the staging or expansion kernels of the
 * same call.  Either may be NULL.  No counterpart in the reference, whose
 * generated wrappers time their one kernel the same way
 * (src/dsl/codegen_cuda.py:257-275). */
int smm_debug_time_next(void* event_before, void* event_after);

/* Failure-path test: the next tensor-core contraction kernel launched from
 * the calling thread gives each pipeline wait `wait_limit_ns` nanoseconds
 * instead of the default (SMM_WAIT_LIMIT_MS, 2000 ms when unset); teardown
 * waits for copies and MMAs already issued keep at least one second.  A limit
 * shorter than the first TMA round trip makes the kernel give up, record
 * the expiry, write no output and exit cleanly; smm_device_status then
 * returns SMM_ERR_DEVICE_TIMEOUT.  0 restores the default; at most 10 s. */
int smm_debug_wait_limit_next(unsigned long long wait_limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* SMM_H */
