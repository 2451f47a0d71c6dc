// Instantiates the tcgen05 GEMM launchers for Arith::TF32.
#include "kx_gemm_launch.cuh"

namespace kx {
int dispatch_gemm_tc_tf32(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                        const GemmParams& p) {
  return dispatch_gemm_tc<Arith::TF32>(bn, amn, bmn, e, pr, p);
}
}  // namespace kx
