// Layout kernels around the implicit-GEMM conv: NCHW <-> NHWC, conv weight packing
// (OIHW -> O,KH,KW,I so the GEMM K index is (tap, channel)), stride-2 parity planes and the
// nearest-neighbour 2x upsample (NHWC).  All are plain HBM-bound copies with 16-byte accesses
// where the channel count allows.
#include <cuda_fp16.h>

#include "common.h"

namespace dlm {

namespace {

// [N, C, HW] -> [N, HW, C] through a 32x32 shared-memory tile.
__global__ void nchw_to_nhwc_kernel(const __half* __restrict__ in, __half* __restrict__ out, int C,
                                    int HW) {
  __shared__ __half tile[32][33];
  const int n = blockIdx.z;
  const int c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
  const __half* src = in + static_cast<size_t>(n) * C * HW;
  __half* dst = out + static_cast<size_t>(n) * C * HW;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, pix = p0 + threadIdx.x;
    if (c < C && pix < HW) tile[i][threadIdx.x] = src[static_cast<size_t>(c) * HW + pix];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int pix = p0 + i, c = c0 + threadIdx.x;
    if (c < C && pix < HW) dst[static_cast<size_t>(pix) * C + c] = tile[threadIdx.x][i];
  }
}

// [N, HW, C] -> [N, C, HW]
__global__ void nhwc_to_nchw_kernel(const __half* __restrict__ in, __half* __restrict__ out, int C,
                                    int HW) {
  __shared__ __half tile[32][33];
  const int n = blockIdx.z;
  const int p0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const __half* src = in + static_cast<size_t>(n) * C * HW;
  __half* dst = out + static_cast<size_t>(n) * C * HW;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int pix = p0 + i, c = c0 + threadIdx.x;
    if (c < C && pix < HW) tile[i][threadIdx.x] = src[static_cast<size_t>(pix) * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, pix = p0 + threadIdx.x;
    if (c < C && pix < HW) dst[static_cast<size_t>(c) * HW + pix] = tile[threadIdx.x][i];
  }
}

// w[o, i, kh, kw] -> p[o, kh, kw, i]
__global__ void pack_conv_weight_kernel(const __half* __restrict__ w, __half* __restrict__ p,
                                        int Cout, int Cin, int KH, int KW) {
  const size_t total = static_cast<size_t>(Cout) * Cin * KH * KW;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    size_t t = idx;
    const int i = static_cast<int>(t % Cin);
    t /= Cin;
    const int kw = static_cast<int>(t % KW);
    t /= KW;
    const int kh = static_cast<int>(t % KH);
    const int o = static_cast<int>(t / KH);
    p[idx] = w[((static_cast<size_t>(o) * Cin + i) * KH + kh) * KW + kw];
  }
}

// x[n, 2h+pr, 2w+pc, c] -> planes[pr*2+pc, n, h, w, c]; C % 8 == 0 (16-byte vectors).
__global__ void parity_planes_kernel(const uint4* __restrict__ x, uint4* __restrict__ planes, int N,
                                     int H, int W, int C8) {
  const int oH = H >> 1, oW = W >> 1;
  const size_t total = static_cast<size_t>(N) * H * W * C8;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    size_t t = idx;
    const int c = static_cast<int>(t % C8);
    t /= C8;
    const int w = static_cast<int>(t % W);
    t /= W;
    const int h = static_cast<int>(t % H);
    const int n = static_cast<int>(t / H);
    const int plane = (h & 1) * 2 + (w & 1);
    const size_t o = (((static_cast<size_t>(plane) * N + n) * oH + (h >> 1)) * oW + (w >> 1)) * C8 + c;
    planes[o] = x[idx];
  }
}

// NHWC nearest 2x: out[n, y, x, c] = in[n, y/2, x/2, c]; C % 8 == 0.
__global__ void upsample2x_nhwc_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, int N,
                                       int H, int W, int C8) {
  const int H2 = H * 2, W2 = W * 2;
  const size_t total = static_cast<size_t>(N) * H2 * W2 * C8;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    size_t t = idx;
    const int c = static_cast<int>(t % C8);
    t /= C8;
    const int x = static_cast<int>(t % W2);
    t /= W2;
    const int y = static_cast<int>(t % H2);
    const int n = static_cast<int>(t / H2);
    out[idx] = in[((static_cast<size_t>(n) * H + (y >> 1)) * W + (x >> 1)) * C8 + c];
  }
}

int grid_for(size_t total, int threads) {
  size_t g = (total + threads - 1) / threads;
  const size_t cap = static_cast<size_t>(num_sms()) * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : static_cast<int>(g);
}

}  // namespace

int nchw_to_nhwc(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s) {
  dim3 grid((HW + 31) / 32, (C + 31) / 32, N), block(32, 8);
  nchw_to_nhwc_kernel<<<grid, block, 0, s>>>(in, out, C, HW);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int nhwc_to_nchw(const __half* in, __half* out, int N, int C, int HW, cudaStream_t s) {
  dim3 grid((C + 31) / 32, (HW + 31) / 32, N), block(32, 8);
  nhwc_to_nchw_kernel<<<grid, block, 0, s>>>(in, out, C, HW);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int pack_conv_weight(const __half* w, __half* p, int Cout, int Cin, int KH, int KW, cudaStream_t s) {
  const size_t total = static_cast<size_t>(Cout) * Cin * KH * KW;
  pack_conv_weight_kernel<<<grid_for(total, 256), 256, 0, s>>>(w, p, Cout, Cin, KH, KW);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int parity_planes(const __half* x, __half* planes, int N, int H, int W, int C, cudaStream_t s) {
  const size_t total = static_cast<size_t>(N) * H * W * (C / 8);
  parity_planes_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      reinterpret_cast<const uint4*>(x), reinterpret_cast<uint4*>(planes), N, H, W, C / 8);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int upsample2x_nhwc(const __half* in, __half* out, int N, int H, int W, int C, cudaStream_t s) {
  const size_t total = static_cast<size_t>(N) * 4 * H * W * (C / 8);
  upsample2x_nhwc_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      reinterpret_cast<const uint4*>(in), reinterpret_cast<uint4*>(out), N, H, W, C / 8);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

}  // namespace dlm
