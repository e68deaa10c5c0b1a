// Contraction kernels with both operands TMA-loaded: dense GEMM and the dense-with-zeros upper-triangular left operand.
#include "smm_launch.cuh"

namespace smm {

int launch_kinds_dense(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Dense && bk == BKind::Dense) return launch_bn<AKind::Dense, BKind::Dense>(bn, pair, mode, m, p, st);
  if (ak == AKind::UpperDense && bk == BKind::Dense) return launch_bn<AKind::UpperDense, BKind::Dense>(bn, pair, mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

}  // namespace smm
