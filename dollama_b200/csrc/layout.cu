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

// p[o, kh, kw, i] (row stride ldp) = w[o, i, kh, kw] for o < Cout, i < Cin; zero for the padding
// rows o in [Cout, Cout_pad) and channels i in [Cin, Cin_pad).
__global__ void pack_conv_pad_kernel(const __half* __restrict__ w, __half* __restrict__ p, int Cout,
                                     int Cout_pad, int Cin, int Cin_pad, int KK, int ldp) {
  const size_t total = static_cast<size_t>(Cout_pad) * KK * Cin_pad;
  for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % Cin_pad);
    const int tap = static_cast<int>((idx / Cin_pad) % KK);
    const int o = static_cast<int>(idx / (static_cast<size_t>(Cin_pad) * KK));
    __half v = __float2half_rn(0.0f);
    if (o < Cout && i < Cin) v = w[(static_cast<size_t>(o) * Cin + i) * KK + tap];
    p[static_cast<size_t>(o) * ldp + static_cast<size_t>(tap) * Cin_pad + i] = v;
  }
}

__global__ void add_f16_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                               __half* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2half_rn(__half2float(a[i]) + __half2float(b[i]));
}

// NCHW [B, Cin, HW] -> NHWC [B, HW, Cpad] with zero channels beyond Cin; one thread per pixel,
// 16-byte stores (Cpad % 8 == 0), reads coalesced across the threads of a warp.
__global__ void nchw_to_nhwc_pad_kernel(const __half* __restrict__ in, __half* __restrict__ out,
                                        int B, int Cin, int HW, int Cpad) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t total = static_cast<size_t>(B) * HW;
  if (i >= total) return;
  const int b = static_cast<int>(i / HW), p = static_cast<int>(i % HW);
  uint4* o = reinterpret_cast<uint4*>(out + i * Cpad);
  for (int c0 = 0; c0 < Cpad; c0 += 8) {
    __align__(16) __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + j;
      h[j] = c < Cin ? in[(static_cast<size_t>(b) * Cin + c) * HW + p] : __float2half_rn(0.0f);
    }
    o[c0 / 8] = *reinterpret_cast<const uint4*>(h);
  }
}

// NHWC [B, HW, ld] (first Cout channels) -> NCHW [B, Cout, HW]
__global__ void nhwc_to_nchw_narrow_kernel(const __half* __restrict__ in, int ld,
                                           __half* __restrict__ out, int B, int Cout, int HW) {
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t total = static_cast<size_t>(B) * HW;
  if (i >= total) return;
  const int b = static_cast<int>(i / HW), p = static_cast<int>(i % HW);
  for (int c = 0; c < Cout; ++c) out[(static_cast<size_t>(b) * Cout + c) * HW + p] = in[i * ld + c];
}

// out[c, s] = in[s * ld + c] for s < S, c < C (32x32 shared tiles)
__global__ void transpose_strided_kernel(const __half* __restrict__ in, int ld, __half* __restrict__ out,
                                         int S, int C) {
  __shared__ __half tile[32][33];
  const int s0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int s = s0 + i, c = c0 + threadIdx.x;
    if (s < S && c < C) tile[i][threadIdx.x] = in[static_cast<size_t>(s) * ld + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, s = s0 + threadIdx.x;
    if (s < S && c < C) out[static_cast<size_t>(c) * S + s] = tile[threadIdx.x][i];
  }
}

// dst[r * cols_p + c] = src[r * rs + c * cs] for r < rows, c < cols; zero in the padding
// (rows_p x cols_p); any strides, so it also transposes
__global__ void gather_pad_kernel(const __half* __restrict__ src, long long rs, long long cs,
                                  int rows, int cols, __half* __restrict__ dst, int rows_p,
                                  int cols_p) {
  const long long total = static_cast<long long>(rows_p) * cols_p;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols_p), c = static_cast<int>(i % cols_p);
    dst[i] = (r < rows && c < cols) ? src[r * rs + c * cs] : __float2half(0.0f);
  }
}

// out = fp16(in * scale), 8 elements per thread (n % 8 == 0)
__global__ void f32_to_f16_scaled_kernel(const float4* __restrict__ in, uint4* __restrict__ out,
                                         size_t n8, float scale) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 a = in[2 * i], b = in[2 * i + 1];
    __half2 h0 = __floats2half2_rn(a.x * scale, a.y * scale);
    __half2 h1 = __floats2half2_rn(a.z * scale, a.w * scale);
    __half2 h2 = __floats2half2_rn(b.x * scale, b.y * scale);
    __half2 h3 = __floats2half2_rn(b.z * scale, b.w * scale);
    out[i] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                        *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}

// NHWC nearest 2x of an fp32 tensor into fp16 scaled by `scale`; C % 8 == 0.
__global__ void upsample2x_f32_to_f16_kernel(const float4* __restrict__ in, uint4* __restrict__ out,
                                             int N, int H, int W, int C8, float scale) {
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
    const size_t src = (((static_cast<size_t>(n) * H + (y >> 1)) * W + (x >> 1)) * C8 + c) * 2;
    const float4 a = in[src], b = in[src + 1];
    __half2 h0 = __floats2half2_rn(a.x * scale, a.y * scale);
    __half2 h1 = __floats2half2_rn(a.z * scale, a.w * scale);
    __half2 h2 = __floats2half2_rn(b.x * scale, b.y * scale);
    __half2 h3 = __floats2half2_rn(b.z * scale, b.w * scale);
    out[idx] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                          *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}

// In-place row softmax of fp16 scores [rows, cols] (already scaled), fp32 arithmetic; one
// 256-thread block per row, the row held in registers (VEC x 8 values per thread, cols <= 2048 VEC).
template <int VEC>
__global__ void __launch_bounds__(256) softmax_rows_kernel(__half* __restrict__ s, int cols) {
  __shared__ float red[8];
  __half* row = s + static_cast<size_t>(blockIdx.x) * cols;
  const int n8 = cols / 8;
  float v[VEC][8];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    const int i = threadIdx.x + 256 * k;
    if (i < n8) {
      const uint4 u = *reinterpret_cast<const uint4*>(row + 8 * i);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(h[q]);
        v[k][2 * q] = f.x;
        v[k][2 * q + 1] = f.y;
        mx = fmaxf(mx, fmaxf(f.x, f.y));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    const int i = threadIdx.x + 256 * k;
    if (i < n8) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[k][q] = __expf(v[k][q] - mx);
        sum += v[k][q];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  sum = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) sum += red[w];
  const float inv = 1.0f / sum;
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    const int i = threadIdx.x + 256 * k;
    if (i < n8) {
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 h = __floats2half2_rn(v[k][2 * q] * inv, v[k][2 * q + 1] * inv);
        o[q] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(row + 8 * i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}
constexpr int kSoftmaxMaxCols = 256 * 8 * 16;

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

int pack_conv_pad(const __half* w, __half* p, int Cout, int Cout_pad, int Cin, int Cin_pad, int KK,
                  int ldp, cudaStream_t s) {
  const size_t total = static_cast<size_t>(Cout_pad) * KK * Cin_pad;
  pack_conv_pad_kernel<<<grid_for(total, 256), 256, 0, s>>>(w, p, Cout, Cout_pad, Cin, Cin_pad, KK, ldp);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int add_f16(const __half* a, const __half* b, __half* y, int n, cudaStream_t s) {
  add_f16_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, b, y, n);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int nchw_to_nhwc_pad(const __half* in, __half* out, int B, int Cin, int HW, int Cpad, cudaStream_t s) {
  DLM_REQUIRE(Cpad % 8 == 0 && Cpad >= Cin && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
              DLM_ERR_INVALID, "nchw_to_nhwc_pad: Cpad=%d must be a multiple of 8 and >= Cin", Cpad);
  const size_t total = static_cast<size_t>(B) * HW;
  nchw_to_nhwc_pad_kernel<<<static_cast<int>((total + 255) / 256), 256, 0, s>>>(in, out, B, Cin, HW, Cpad);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int nhwc_to_nchw_narrow(const __half* in, int ld, __half* out, int B, int Cout, int HW, cudaStream_t s) {
  const size_t total = static_cast<size_t>(B) * HW;
  nhwc_to_nchw_narrow_kernel<<<static_cast<int>((total + 255) / 256), 256, 0, s>>>(in, ld, out, B, Cout, HW);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int transpose_strided(const __half* in, int ld, __half* out, int S, int C, cudaStream_t s) {
  dim3 grid((S + 31) / 32, (C + 31) / 32), block(32, 8);
  transpose_strided_kernel<<<grid, block, 0, s>>>(in, ld, out, S, C);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int gather_pad(const __half* src, long long rs, long long cs, int rows, int cols, __half* dst,
               int rows_p, int cols_p, cudaStream_t s) {
  const long long total = static_cast<long long>(rows_p) * cols_p;
  if (total == 0) return DLM_OK;
  gather_pad_kernel<<<grid_for(static_cast<size_t>(total), 256), 256, 0, s>>>(src, rs, cs, rows, cols,
                                                                             dst, rows_p, cols_p);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int f32_to_f16_scaled(const float* in, __half* out, size_t n, float scale, cudaStream_t s) {
  DLM_REQUIRE(n % 8 == 0, DLM_ERR_INVALID, "f32_to_f16_scaled: n %% 8");
  f32_to_f16_scaled_kernel<<<grid_for(n / 8, 256), 256, 0, s>>>(
      reinterpret_cast<const float4*>(in), reinterpret_cast<uint4*>(out), n / 8, scale);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int upsample2x_f32_to_f16(const float* in, __half* out, int N, int H, int W, int C, float scale,
                          cudaStream_t s) {
  DLM_REQUIRE(C % 8 == 0, DLM_ERR_INVALID, "upsample2x_f32_to_f16: C %% 8");
  const size_t total = static_cast<size_t>(N) * 4 * H * W * (C / 8);
  upsample2x_f32_to_f16_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      reinterpret_cast<const float4*>(in), reinterpret_cast<uint4*>(out), N, H, W, C / 8, scale);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int softmax_rows_f16(__half* s_, int rows, int cols, cudaStream_t s) {
  DLM_REQUIRE(cols % 8 == 0 && cols <= kSoftmaxMaxCols, DLM_ERR_INVALID,
              "softmax_rows: cols=%d must be a multiple of 8 and <= %d", cols, kSoftmaxMaxCols);
  const int vec = (cols / 8 + 255) / 256;
  if (vec <= 1)
    softmax_rows_kernel<1><<<rows, 256, 0, s>>>(s_, cols);
  else if (vec <= 2)
    softmax_rows_kernel<2><<<rows, 256, 0, s>>>(s_, cols);
  else if (vec <= 4)
    softmax_rows_kernel<4><<<rows, 256, 0, s>>>(s_, cols);
  else if (vec <= 8)
    softmax_rows_kernel<8><<<rows, 256, 0, s>>>(s_, cols);
  else
    softmax_rows_kernel<16><<<rows, 256, 0, s>>>(s_, cols);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

}  // namespace dlm
