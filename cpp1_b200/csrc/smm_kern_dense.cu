// Contraction kernels with both operands TMA-loaded: dense GEMM and the dense-with-zeros upper-triangular
// left operand (both also split along K over CTA clusters for products with few output tiles).
#include "smm_launch.cuh"

namespace smm {

int launch_kinds_dense(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Dense && bk == BKind::Dense) return launch_bn<AKind::Dense, BKind::Dense>(bn, pair, mode, m, p, st);
  if (ak == AKind::UpperDense && bk == BKind::Dense) return launch_bn<AKind::UpperDense, BKind::Dense>(bn, pair, mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

template <AKind A>
int launch_split(int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  constexpr BKind B = BKind::Dense;
  if (mode == SMM_MODE_3XTF32)
    return launch_umma<A, B, Mode::TF32x3, 128, umma_stages<A, Mode::TF32x3, 128>(), false, 2>(m, p, st);
  if (mode == SMM_MODE_BF16)
    return launch_umma<A, B, Mode::BF16, 128, umma_stages<A, Mode::BF16, 128>(), false, 2>(m, p, st);
  return launch_umma<A, B, Mode::TF32, 128, umma_stages<A, Mode::TF32, 128>(), false, 2>(m, p, st);
}

int launch_dense_split(AKind ak, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Dense) return launch_split<AKind::Dense>(mode, m, p, st);
  if (ak == AKind::UpperDense) return launch_split<AKind::UpperDense>(mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "split-K contraction: unsupported operand kinds");
}

int launch_dense_persist(AKind ak, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Dense)
    return mode == SMM_MODE_BF16 ? launch_persist<AKind::Dense, Mode::BF16>(m, p, st)
                                 : launch_persist<AKind::Dense, Mode::TF32>(m, p, st);
  if (ak == AKind::UpperDense)
    return mode == SMM_MODE_BF16 ? launch_persist<AKind::UpperDense, Mode::BF16>(m, p, st)
                                 : launch_persist<AKind::UpperDense, Mode::TF32>(m, p, st);
  return set_error(SMM_ERR_INVALID, "persistent contraction: unsupported operand kinds");
}

}  // namespace smm
