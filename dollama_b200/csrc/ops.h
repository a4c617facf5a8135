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

}  // namespace dlm
