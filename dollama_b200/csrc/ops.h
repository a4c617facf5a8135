// Internal (C++) launchers shared by the C-ABI wrappers and the model graphs.
#pragma once

#include <cuda_fp16.h>

#include "common.h"

namespace dlm {

// layout.cu
int nchw_to_nhwc(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s);
int nhwc_to_nchw(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s);
int pack_conv_weight(const __half* w, __half* p, int Cout, int Cin, int KH, int KW, cudaStream_t s);
int parity_planes(const __half* x, __half* planes, int N, int H, int W, int C, cudaStream_t s);
int upsample2x_nhwc(const __half* in, __half* out, int N, int H, int W, int C, cudaStream_t s);
// p[o, tap, i] (row stride ldp) from OIHW w, zero rows o >= Cout and channels i >= Cin.
int pack_conv_pad(const __half* w, __half* p, int Cout, int Cout_pad, int Cin, int Cin_pad, int KK,
                  int ldp, cudaStream_t s);
// y = fp16(a + b), n elements (weight preparation)
int add_f16(const __half* a, const __half* b, __half* y, int n, cudaStream_t s);
int nchw_to_nhwc_pad(const __half* in, __half* out, int B, int Cin, int HW, int Cpad, cudaStream_t s);
int nhwc_to_nchw_narrow(const __half* in, int ld, __half* out, int B, int Cout, int HW, cudaStream_t s);
int transpose_strided(const __half* in, int ld, __half* out, int S, int C, cudaStream_t s);
// dst [rows_p, cols_p] = src(r, c) = src[r * rs + c * cs] inside [rows, cols], zero outside
int gather_pad(const __half* src, long long rs, long long cs, int rows, int cols, __half* dst,
               int rows_p, int cols_p, cudaStream_t s);
int f32_to_f16_scaled(const float* in, __half* out, size_t n, float scale, cudaStream_t s);
int upsample2x_f32_to_f16(const float* in, __half* out, int N, int H, int W, int C, float scale,
                          cudaStream_t s);
int softmax_rows_f16(__half* s_, int rows, int cols, cudaStream_t s);

}  // namespace dlm
