// gemm_s8.cu — s8 × s8 → s32 tcgen05 GEMM instantiations (futon's Q8 path).
#include "gemm_launch.cuh"

namespace futon {
cudaError_t launch_gemm_s8(const GemmLaunch& g) { return launch_gemm_any<true, false>(g); }
}  // namespace futon
