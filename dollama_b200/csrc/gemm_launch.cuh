// Launchers of the tcgen05 GEMM kernels for one compile-time epilogue flag set FL (see kEpiDyn in
// gemm_tc.cuh).  Each FL's kernels are instantiated in one translation unit (gemm_fl*.cu for the
// flag sets the model handles use, gemm.cu for the run-time generic path) so that the units
// compile in parallel; gemm_launch picks the instantiation from the op's flags.
#pragma once

#include "gemm.h"
#include "ops.h"

namespace dlm {

template <int BN, unsigned FL>
int launch_bn(const GemmOp& op, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm_smem_bytes(BN);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, FL>, op.tmA[0], op.tmA[1], op.tmA[2],
                                    op.tmB, op.tmC, op.p));
  return DLM_OK;
}

template <int BN, unsigned FL>
int launch_bn2(const GemmOp& op, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm2_smem_bytes(BN);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<BN, FL>, op.tmA[0], op.tmA[1], op.tmA[2],
                                    op.tmB, op.tmC, op.p));
  return DLM_OK;
}

// Dynamic shared-memory limits of every tile variant of this FL (set before any launch, so that
// no attribute call happens inside a CUDA-graph capture).
template <unsigned FL>
int gemm_prepare_fl() {
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<256, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(256)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<192, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(192)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<160, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(160)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<128, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(128)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<64, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(64)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<256, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2_smem_bytes(256)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<224, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2_smem_bytes(224)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<192, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2_smem_bytes(192)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<160, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2_smem_bytes(160)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<128, FL>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm2_smem_bytes(128)));
  return DLM_OK;
}

template <unsigned FL>
int gemm_launch_fl(const GemmOp& op, cudaStream_t s) {
  if (op.pair) {
    switch (op.bn) {
      case 256: return launch_bn2<256, FL>(op, s);
      case 224: return launch_bn2<224, FL>(op, s);
      case 192: return launch_bn2<192, FL>(op, s);
      case 160: return launch_bn2<160, FL>(op, s);
      case 128: return launch_bn2<128, FL>(op, s);
      default: break;
    }
  } else {
    switch (op.bn) {
      case 256: return launch_bn<256, FL>(op, s);
      case 192: return launch_bn<192, FL>(op, s);
      case 160: return launch_bn<160, FL>(op, s);
      case 128: return launch_bn<128, FL>(op, s);
      case 64: return launch_bn<64, FL>(op, s);
      default: break;
    }
  }
  set_error("gemm: op not planned");
  return DLM_ERR_INVALID;
}

// The flag sets with their own instantiations: every epilogue the UNet step plans
// (bias / residual / row statistics / LayerNorm fold / GEGLU / per-image bias / SiLU).
#define DLM_GEMM_SPECIAL_FLAGS(X)                                                                  \
  X(0x000u) X(0x001u) X(0x003u) X(0x009u) X(0x010u) X(0x101u) X(0x103u) X(0x200u) X(0x204u)

#define DLM_GEMM_DECLARE_FL(F)                                                                     \
  extern template int gemm_launch_fl<F>(const GemmOp&, cudaStream_t);                             \
  extern template int gemm_prepare_fl<F>();
DLM_GEMM_SPECIAL_FLAGS(DLM_GEMM_DECLARE_FL)
#undef DLM_GEMM_DECLARE_FL

#define DLM_GEMM_INSTANTIATE_FL(F)                                                                 \
  template int gemm_launch_fl<F>(const GemmOp&, cudaStream_t);                                     \
  template int gemm_prepare_fl<F>();

}  // namespace dlm
