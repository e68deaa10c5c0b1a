// Contraction kernels with a Toeplitz left operand expanded from its generator on chip.
#include "smm_launch.cuh"

namespace smm {

int launch_kinds_toeplitz(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Toeplitz && bk == BKind::Dense) return launch_bn<AKind::Toeplitz, BKind::Dense>(bn, pair, mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

}  // namespace smm
