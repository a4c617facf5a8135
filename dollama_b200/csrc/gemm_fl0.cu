// GEMM kernel instantiations for the epilogue flag sets 0x000u 0x001u 0x003u (compiled as their own unit).
#include "gemm_launch.cuh"

namespace dlm {
DLM_GEMM_INSTANTIATE_FL(0x000u)
DLM_GEMM_INSTANTIATE_FL(0x001u)
DLM_GEMM_INSTANTIATE_FL(0x003u)
}  // namespace dlm
