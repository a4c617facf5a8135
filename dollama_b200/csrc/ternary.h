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
// value (one float add) instead.
int ternary_gemm_i8(const uint32_t* wp, const float* alpha, const int8_t* xq, const float* xscale,
                    float* y, int M, int N, int K, cudaStream_t s, bool accumulate = false);

}  // namespace dlm
