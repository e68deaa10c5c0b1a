// Contraction kernels with a structured right operand built on chip (the DSL's Gen@Upper, Gen@Symm, Gen@Lower, Gen@Toeplitz, Symm@Symm, Lower@Lower).
#include "smm_launch.cuh"

namespace smm {

int launch_kinds_right(AKind ak, BKind bk, int bn, bool pair, int mode, const Maps& m, const UmmaParams& p, cudaStream_t st) {
  if (ak == AKind::Dense && bk == BKind::UpperPacked) return launch_bn<AKind::Dense, BKind::UpperPacked>(bn, pair, mode, m, p, st);
  if (ak == AKind::Dense && bk == BKind::SymmPacked) return launch_bn<AKind::Dense, BKind::SymmPacked>(bn, pair, mode, m, p, st);
  if (ak == AKind::Dense && bk == BKind::Toeplitz) return launch_bn<AKind::Dense, BKind::Toeplitz>(bn, pair, mode, m, p, st);
  if (ak == AKind::Dense && bk == BKind::LowerPacked) return launch_bn<AKind::Dense, BKind::LowerPacked>(bn, pair, mode, m, p, st);
  if (ak == AKind::SymmPacked && bk == BKind::SymmPacked) return launch_bn<AKind::SymmPacked, BKind::SymmPacked>(bn, pair, mode, m, p, st);
  if (ak == AKind::LowerPacked && bk == BKind::LowerPacked) return launch_bn<AKind::LowerPacked, BKind::LowerPacked>(bn, pair, mode, m, p, st);
  return set_error(SMM_ERR_INVALID, "unsupported operand kinds");
}

}  // namespace smm
