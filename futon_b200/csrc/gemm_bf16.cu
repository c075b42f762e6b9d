// gemm_bf16.cu — bf16 × bf16 → f32 tcgen05 GEMM instantiations (the MatMulT seam).
#include "gemm_launch.cuh"

namespace futon {
cudaError_t launch_gemm_bf16(const GemmLaunch& g) { return launch_gemm_any<false, false>(g); }
}  // namespace futon
