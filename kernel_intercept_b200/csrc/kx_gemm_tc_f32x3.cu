// Instantiates the tcgen05 GEMM launchers for Arith::F32x3.
#include "kx_gemm_launch.cuh"

namespace kx {
int dispatch_gemm_tc_f32x3(int bn, bool amn, bool bmn, const Exec& e, const TcProblem& pr,
                        const GemmParams& p) {
  return dispatch_gemm_tc<Arith::F32x3>(bn, amn, bmn, e, pr, p);
}
}  // namespace kx
