// Tensor-core 3xTF32 GEMM for sm_100a (tcgen05 + TMEM + TMA).
// Placeholder until the kernel lands: every problem is reported unsupported so
// mtc_matmul's AUTO mode takes the exact SIMT path.
#include "gemm.cuh"

namespace mtc {

int gemm_3xtf32(const GemmProblem &, cudaStream_t) {
    return fail(MTC_ERR_UNSUPPORTED, "tensor-core 3xTF32 GEMM not built");
}

}  // namespace mtc
