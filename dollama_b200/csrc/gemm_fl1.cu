// GEMM kernel instantiations for the epilogue flag sets 0x009u 0x010u 0x101u (compiled as their own unit).
#include "gemm_launch.cuh"

namespace dlm {
DLM_GEMM_INSTANTIATE_FL(0x009u)
DLM_GEMM_INSTANTIATE_FL(0x010u)
DLM_GEMM_INSTANTIATE_FL(0x101u)
}  // namespace dlm
