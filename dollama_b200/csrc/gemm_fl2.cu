// GEMM kernel instantiations for the epilogue flag sets 0x103u 0x200u 0x204u (compiled as their own unit).
#include "gemm_launch.cuh"

namespace dlm {
DLM_GEMM_INSTANTIATE_FL(0x103u)
DLM_GEMM_INSTANTIATE_FL(0x200u)
DLM_GEMM_INSTANTIATE_FL(0x204u)
}  // namespace dlm
