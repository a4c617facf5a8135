// Host-side planning / launching of the tcgen05 GEMM (dense linear and implicit-GEMM conv).
#pragma once

#include <cuda_fp16.h>

#include "common.h"
#include "gemm_tc.cuh"

namespace dlm {

// A fully-encoded GEMM launch: tensor maps + kernel parameters.  Built once, launched many
// times (the UNet builds all of its ops at plan time and replays them in a CUDA graph).
struct GemmOp {
  CUtensorMap tmA[3];
  CUtensorMap tmB;
  CUtensorMap tmC;  // output, 32-row boxes for the staged epilogue stores
  GemmParams p;
  int bn = 0;
  bool pair = false;  // CTA-pair (cta_group::2) kernel
  int grid = 0;
  long long k_true = 0;  // reduction length before padding to 64 (host-side bookkeeping)
};

struct GemmEpilogue {
  unsigned flags = 0;
  float alpha = 1.0f;
  float resid_scale = 1.0f;
  const __half* bias = nullptr;
  const __half* bias2d = nullptr;
  int rows_per_img = 1;
  int ldb2 = 0;  // row stride of bias2d (0 = N)
  const __half* resid = nullptr;
  int ldr = 0;
  // internal modes (kEpiRowStats / kEpiLnFold in flags)
  float2* stats_out = nullptr;      // [M, n_tiles] (mean, M2) per row and N tile of the output
  const float2* stats_in = nullptr; // producer statistics of the A operand rows
  int stats_in_parts = 0, stats_in_tile = 0, ln_C = 0;
  float ln_eps = 1e-5f;
  const float* ln_u = nullptr;      // [N] sum_k W'[n,k]
  const float* ln_v = nullptr;      // [N] sum_k beta[k] W[n,k] + bias[n]
  // stream-K workspace (optional): gemm_sk_workspace_bytes() bytes whose first
  // gemm_sk_flag_bytes() are zero before the first launch (every launch leaves them zero).  When
  // present, the planner may split the k-block iterations of a launch with fewer tiles than SMs
  // over all SMs.  Launches sharing a workspace must not overlap on the GPU.
  void* sk_ws = nullptr;
  size_t sk_ws_bytes = 0;
};

// One source of an implicit-GEMM conv K segment.
struct ConvSource {
  int kind = 0;               // 0: 3x3 s1, 1: 1x1, 2: 3x3 s2 from parity planes
  const __half* ptr = nullptr; // NHWC [Nb, oH, oW, C] (kinds 0/1) or planes [4, Nb, oH, oW, C]
  int C = 0;                  // channels, multiple of 64
};

// Dense: C[M, ldc] = epi(A[M, K] (row stride lda) * W[N, K]^T).
int gemm_plan_dense(GemmOp* op, const __half* A, int lda, const __half* W, int M, int N, int K,
                    __half* C, int ldc, const GemmEpilogue& epi, int force_bn = 0, int ldw = 0);

// Implicit-GEMM conv producing NHWC out[Nb, oH, oW, Cout] (row stride ldc) from up to three
// K segments; W is [Cout, sum(taps_s * C_s)] with the K index ordered (segment, tap, channel).
int gemm_plan_conv(GemmOp* op, int Nb, int oH, int oW, const ConvSource* srcs, int nsrc,
                   const __half* W, int Cout, __half* C, int ldc, const GemmEpilogue& epi,
                   int force_bn = 0);

int gemm_launch(const GemmOp& op, cudaStream_t stream);

// Size of a stream-K workspace for this device, and of its flag head (zero between launches).
size_t gemm_sk_workspace_bytes();
size_t gemm_sk_flag_bytes();

// Sets kernel attributes of every variant on the current device (call before graph capture).
int gemm_prepare_kernels();

}  // namespace dlm
