// Ternary-weight x int8-activation linear (BitLinear) launchers, shared by the C ABI and the LM.
#pragma once

#include <cstdint>

#include "common.h"

namespace dlm {

// Per-output-row absmean ternary quantization + 2-bit packing of w [N, K] (K % 64 == 0).
int ternary_pack(const float* w, int N, int K, uint32_t* packed, float* alpha, cudaStream_t s);
// The same rule with ONE alpha for the whole tensor (alpha[n] all equal).
int ternary_pack_per_tensor(const float* w, int N, int K, uint32_t* packed, float* alpha,
                            double* scratch, cudaStream_t s);
// Per-token absmax int8 quantization of x [M, K].
int quantize_act_i8(const float* x, int M, int K, int8_t* xq, float* xscale, cudaStream_t s);
// y [M, N] = float(double(int32 sum) * alpha[n] * xscale[m]); with `accumulate`, y += that
// value (one float add) instead.  `weights_resident`: no kernel still queued or running in the
// stream writes wp / alpha, so a decode-sized call may read them before the previous kernel ends.
int ternary_gemm_i8(const uint32_t* wp, const float* alpha, const int8_t* xq, const float* xscale,
                    float* y, int M, int N, int K, cudaStream_t s, bool accumulate = false,
                    bool weights_resident = false);

// Token rows from which ternary_gemm_i8 uses the tensor cores.
int ternary_tc_min_rows();

// The LM's decode q|k|v projection (one position per sequence, N = 3 D) with RoPE and the K / V
// cache append in its epilogue: row m is sequence m at position *pos; output columns [0, D) are q
// (rotated, to q[m][D]), [D, 2D) k (rotated, into kc), [2D, 3D) v (into vc); caches
// [M][D / 64][Lmax][64]; cos_t / sin_t [position][32].  Same operations, in the same order, as
// the projection followed by the separate RoPE kernel.
struct RopeQkv {
  const int* pos;
  const double* cos_t;
  const double* sin_t;
  float* q;
  float* kc;
  float* vc;
  int D, Lmax;
};
int ternary_gemm_qkv_rope(const uint32_t* wp, const float* alpha, const int8_t* xq,
                          const float* xscale, int M, int K, const RopeQkv& r, cudaStream_t s,
                          bool weights_resident = false);

}  // namespace dlm
