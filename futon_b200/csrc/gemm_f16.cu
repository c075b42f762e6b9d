// gemm_f16.cu — f16 × f16 → f32 tcgen05 GEMM instantiations with every
// epilogue of the forward (the float path computes with f16 operands).
#include "gemm_launch.cuh"

namespace futon {
cudaError_t launch_gemm_f16(const GemmLaunch& g) { return launch_gemm_any<false, true>(g); }
}  // namespace futon
