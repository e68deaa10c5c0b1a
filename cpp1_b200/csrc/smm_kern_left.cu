// Contraction kernels with a packed triangular / symmetric left operand built on chip.
#include "smm_launch.cuh"

namespace smm {

int launch_kinds_left(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::UpperPacked && bk == BKind::Dense) return launch_bn<AKind::UpperPacked, BKind::Dense>(bn, pair, mode, m, p, st);
  if (ak == AKind::SymmPacked && bk == BKind::Dense) return launch_bn<AKind::SymmPacked, BKind::Dense>(bn, pair, mode, m, p, st);
  if (ak == AKind::LowerPacked && bk == BKind::Dense) return launch_bn<AKind::LowerPacked, BKind::Dense>(bn, pair, mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

}  // namespace smm
