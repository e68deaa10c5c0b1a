// Launch templates of the contraction engine and the per-operand-kind
// launchers.  Each operand pairing is instantiated in its own translation
// unit (smm_kern_*.cu), so the kernel variants compile in parallel.
#pragma once
#include <cuda.h>
#include <algorithm>
#include <cuda_runtime.h>

#include "smm_host.h"
#include "smm_umma.cuh"
#include "smm_umma_persist.cuh"

namespace smm {

struct Maps {
  CUtensorMap a{}, b{}, al{}, bl{};
};

template <AKind AK, BKind BK, Mode MD, int BN, int STAGES, bool PAIR, int SPLITK = 1>
int launch_umma(const Maps& m, const UmmaParams& p, cudaStream_t st) {
  auto kern = umma_gemm_kernel<AK, BK, MD, BN, STAGES, PAIR, SPLITK>;
  constexpr int kCluster = PAIR ? 2 : SPLITK;
  constexpr int smem = umma_smem_bytes<AK, MD, PAIR ? BN / 2 : BN, STAGES>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static bool attr_set[64] = {};
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {  // cached for device indices below 64
    SMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute(max dynamic smem)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const long long blocks = static_cast<long long>(p.row_tiles) * p.col_tiles * kCluster;
  if (blocks > 0x7FFFFFFFLL) return set_error(SMM_ERR_INVALID, "product too large for one launch");
  if constexpr (kCluster > 1) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
    cfg.blockDim = dim3(umma_threads(AK, MD), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, m.a, m.b, m.al, m.bl, p), "tcgen05 cluster contraction launch");
  } else {
    kern<<<static_cast<unsigned>(blocks), umma_threads(AK, MD), smem, st>>>(m.a, m.b, m.al, m.bl, p);
  }
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "tcgen05 contraction launch");
  return SMM_OK;
}

// Stage counts fill ~192 KiB of shared memory (umma_stages).
template <AKind AK, BKind BK, int BN, bool PAIR>
int launch_mode(int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  constexpr int kCols = PAIR ? BN / 2 : BN;  // B columns per CTA
  if (mode == SMM_MODE_3XTF32)
    return launch_umma<AK, BK, Mode::TF32x3, BN, umma_stages<AK, Mode::TF32x3, kCols>(), PAIR>(m, p, st);
  if (mode == SMM_MODE_BF16)
    return launch_umma<AK, BK, Mode::BF16, BN, umma_stages<AK, Mode::BF16, kCols>(), PAIR>(m, p, st);
  return launch_umma<AK, BK, Mode::TF32, BN, umma_stages<AK, Mode::TF32, kCols>(), PAIR>(m, p, st);
}

template <AKind AK, BKind BK>
int launch_bn(int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (pair) {
    if (bn == 256) return launch_mode<AK, BK, 256, true>(mode, m, p, st);
    return launch_mode<AK, BK, 128, true>(mode, m, p, st);
  }
  switch (bn) {
    case 256: return launch_mode<AK, BK, 256, false>(mode, m, p, st);
    case 128: return launch_mode<AK, BK, 128, false>(mode, m, p, st);
    default: return launch_mode<AK, BK, 64, false>(mode, m, p, st);
  }
}

// Persistent pair kernel (one-pass modes, TMA-fed A and B, 256 x 256 tiles):
// one cluster per SM pair, at most one per tile.
template <AKind AK, Mode MD>
int launch_persist(const Maps& m, const UmmaParams& p, cudaStream_t st) {
  auto kern = umma_persist_kernel<AK, MD>;
  constexpr int smem = persist_smem_bytes<AK, MD>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static bool attr_set[64] = {};
  int dev = 0;
  SMM_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    SMM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                 "cudaFuncSetAttribute(max dynamic smem)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  int sms = 0;
  SMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
  const long long tiles = static_cast<long long>(p.row_tiles) * p.col_tiles;
  const long long clusters = std::min<long long>(tiles, std::max(1, sms / 2));
  if (clusters <= 0) return SMM_OK;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
  cfg.blockDim = dim3(kPersistThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  SMM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, m.a, m.b, p), "tcgen05 persistent contraction launch");
  count_launch();
  SMM_CUDA_TRY(cudaGetLastError(), "tcgen05 persistent contraction launch");
  return SMM_OK;
}
// Dense / UpperDense x Dense, TF32 or bf16 (smm_kern_dense.cu).
int launch_dense_persist(AKind ak, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st);

// Dense / UpperDense x Dense with 128 x 128 tiles, each split over two CTAs
// along K (smm_kern_dense.cu).
int launch_dense_split(AKind ak, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st);

// One launcher per translation unit; each returns SMM_ERR_INVALID for
// pairings it does not hold.
int launch_kinds_dense(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p,
                       cudaStream_t st);  // smm_kern_dense.cu
int launch_kinds_left(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p,
                      cudaStream_t st);  // smm_kern_left.cu
int launch_kinds_toeplitz(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p,
                          cudaStream_t st);  // smm_kern_toeplitz.cu
int launch_kinds_right(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p,
                       cudaStream_t st);  // smm_kern_right.cu

inline int launch_kinds(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p,
                        cudaStream_t st) {
  if (bk == BKind::Dense) {
    if (ak == AKind::Dense || ak == AKind::UpperDense) return launch_kinds_dense(ak, bk, bn, pair, mode, m, p, st);
    if (ak == AKind::Toeplitz) return launch_kinds_toeplitz(ak, bk, bn, pair, mode, m, p, st);
    return launch_kinds_left(ak, bk, bn, pair, mode, m, p, st);
  }
  return launch_kinds_right(ak, bk, bn, pair, mode, m, p, st);
}

}  // namespace smm
