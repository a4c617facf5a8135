// GroupNorm (NHWC, optional two-source concat + SiLU) and LayerNorm launchers (norm.cu).
#pragma once

#include <cuda_fp16.h>

#include "common.h"

namespace dlm {

struct GnOp {
  const float* xf = nullptr;  // fp32 single-source input (then x1 / x2 are unused)
  const __half* x1 = nullptr;
  const __half* x2 = nullptr;
  int C1 = 0, C2 = 0, N = 0, HW = 0;
  const __half* gamma = nullptr;
  const __half* beta = nullptr;
  float eps = 1e-5f;
  bool silu = false;
  __half* out = nullptr;
  float2* partials = nullptr;   // [N, chunks, 32] (sum, sum of squares)
  float2* mean_rstd = nullptr;  // [N, 32] written by the last statistics block of each image
  unsigned* counters = nullptr; // [N] arrival counters; zero between launches
  int chunks = 0, pix_per_chunk = 0, pix_per_block = 0, stat_smem = 0;
};

// out[N, HW, C1 + C2] = GN32(concat(x1[N, HW, C1], x2[N, HW, C2])) (+ SiLU); `partials` is a
// scratch buffer of at least gn_partial_elems(N, HW) float2 whose arrival counters (op.counters,
// gn_counter_bytes(N)) are zero before the first launch; every launch leaves them at zero.
int gn_plan(GnOp* op, const __half* x1, int C1, const __half* x2, int C2, int N, int HW,
            const __half* gamma, const __half* beta, float eps, bool silu, __half* out,
            float2* partials, size_t partial_cap);
// Same with an fp32 input [N, HW, C] (single source).
int gn_plan_f32(GnOp* op, const float* x, int C, int N, int HW, const __half* gamma,
                const __half* beta, float eps, bool silu, __half* out, float2* partials,
                size_t partial_cap);
size_t gn_partial_elems(int N, int HW);
size_t gn_counter_bytes(int N);
int gn_launch(const GnOp& op, cudaStream_t s);

int layer_norm(const __half* x, const __half* gamma, const __half* beta, __half* out, int rows, int C,
               float eps, cudaStream_t s);

}  // namespace dlm
