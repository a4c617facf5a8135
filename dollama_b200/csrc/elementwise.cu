// The reference kernel library's small host functions, with the reference's layouts and rounding
// sequences, for callers outside this library's fused model graphs (the UNet / VAE handles fold
// all of these into their GEMM epilogues and never call them).
//
//   dlm_bias_add_rowvec      src/kernels/bias_add.cuh:32  out[t,c] = h(f(in[t,c]) + f(bias[c]))
//   dlm_bias_add_channel     src/kernels/bias_add.cuh:51  NCHW, out = h(f(in) + f(bias[c]))
//   dlm_conv_bias_biasch     src/kernels/bias_add.cuh:75  t = h(f(conv) + f(cb[c]));
//                                                          out = h(f(t) + f(tproj[n, c]))
//   dlm_conv_bias_residual   src/kernels/bias_add.cuh:96  t = h(f(conv) + f(cb[c]));
//                                                          out = h(f(t) + f(res))
//   dlm_silu / dlm_gelu / dlm_gelu_tanh  src/kernels/activation.cuh:33-41 (fp32 math)
//   dlm_add                  src/kernels/elementwise.cuh:26  out = h(f(a) + f(b))
//   dlm_upsample_nearest2x   src/kernels/elementwise.cuh:37  NCHW [N,C,H,W] -> [N,C,2H,2W]
//   dlm_geglu                src/kernels/geglu.cuh:42  [tokens, 2d] -> [tokens, d],
//                                                        x1 * gelu_erf(x2), x1 = first half
//   dlm_timestep_embedding   src/kernels/timeembed.cuh:44  [cos(t f_i) | sin(t f_i)],
//                                                          f_i = exp(-ln(max_period) i / half)
//   dlm_gemm_f32             src/kernels/gemm.cuh:61  fp32 row-major C = a op(A) op(B) + b C
//
// h() = round to fp16, f() = widen to fp32.  Each is one HBM pass (the f32 GEMM excepted); all
// return DLM_OK without launching for empty sizes, as the reference's wrappers return.
#include <cuda_fp16.h>

#include "common.h"

namespace dlm {
namespace {

constexpr int kThreads = 256;

inline int blocks_for(long long n) {
  const long long b = (n + kThreads - 1) / kThreads;
  return static_cast<int>(b < 65535LL * 64 ? b : 65535LL * 64);
}

__global__ void bias_rowvec_kernel(const __half* __restrict__ in, const __half* __restrict__ bias,
                                   __half* __restrict__ out, long long n, int C) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = __float2half(__half2float(in[i]) + __half2float(bias[i % C]));
}

__global__ void bias_channel_kernel(const __half* __restrict__ in, const __half* __restrict__ bias,
                                    __half* __restrict__ out, long long n, int C, int HW) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>((i / HW) % C);
    out[i] = __float2half(__half2float(in[i]) + __half2float(bias[c]));
  }
}

// mode 0: second term per (n, c) from tproj[n * C + c]; mode 1: per element from res[i]
__global__ void conv_bias_two_kernel(const __half* __restrict__ conv, const __half* __restrict__ cb,
                                     const __half* __restrict__ second, __half* __restrict__ out,
                                     long long n, int C, int HW, int mode) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long nc = i / HW;
    const int c = static_cast<int>(nc % C);
    const __half t = __float2half(__half2float(conv[i]) + __half2float(cb[c]));
    const __half s2 = mode == 0 ? second[nc] : second[i];
    out[i] = __float2half(__half2float(t) + __half2float(s2));
  }
}

// kind 0 SiLU (x * 1 / (1 + e^-x), fast exp), 1 GELU (erf), 2 GELU (tanh approximation)
__global__ void activation_kernel(const __half* __restrict__ in, __half* __restrict__ out, long long n,
                                  int kind) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = __half2float(in[i]);
    float y;
    if (kind == 0) {
      y = x * (1.0f / (1.0f + __expf(-x)));
    } else if (kind == 1) {
      y = 0.5f * x * (1.0f + erff(x * 0.70710678f));
    } else {
      const float inner = 0.7978845608f * (x + 0.044715f * x * x * x);
      y = 0.5f * x * (1.0f + tanhf(inner));
    }
    out[i] = __float2half(y);
  }
}

__global__ void add_kernel(const __half* __restrict__ a, const __half* __restrict__ b,
                           __half* __restrict__ out, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = __float2half(__half2float(a[i]) + __half2float(b[i]));
}

__global__ void upsample_nchw_kernel(const __half* __restrict__ in, __half* __restrict__ out,
                                     long long n_out, int H, int W) {
  const int W2 = 2 * W, H2 = 2 * H;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n_out;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % W2);
    const long long r = i / W2;
    const int y = static_cast<int>(r % H2);
    const long long plane = r / H2;
    out[i] = in[(plane * H + (y >> 1)) * W + (x >> 1)];
  }
}

__global__ void geglu_kernel(const __half* __restrict__ in, __half* __restrict__ out, long long n, int d) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / d;
    const int c = static_cast<int>(i - t * d);
    const float x1 = __half2float(in[t * 2 * d + c]);
    const float x2 = __half2float(in[t * 2 * d + d + c]);
    const float g = 0.5f * x2 * (1.0f + erff(x2 * 0.70710678f));
    out[i] = __float2half(x1 * g);
  }
}

__global__ void timestep_embedding_kernel(__half* __restrict__ out, float timestep, int half,
                                          float log_max_period) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= half) return;
  const float exponent = -log_max_period * static_cast<float>(i) / static_cast<float>(half);
  const float arg = timestep * __expf(exponent);
  out[i] = __float2half(cosf(arg));
  out[half + i] = __float2half(sinf(arg));
}

// fp32 GEMM, 64 x 64 output tile per 256-thread block (4 x 4 per thread), 16-deep k slices in
// shared memory; op(A)[m, k] = transA ? A[k * M + m] : A[m * K + k], likewise B ([K, N] or [N, K]).
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       float* __restrict__ C, int M, int N, int K,
                                                       float alpha, float beta, int transA, int transB) {
  __shared__ float sa[16][64 + 1];
  __shared__ float sb[16][64 + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      const int kk = e >> 6, mm = e & 63;
      const int m = m0 + mm, k = k0 + kk;
      float va = 0.0f, vb = 0.0f;
      if (m < M && k < K) va = transA ? A[static_cast<size_t>(k) * M + m] : A[static_cast<size_t>(m) * K + k];
      const int nn = n0 + mm;
      if (nn < N && k < K) vb = transB ? B[static_cast<size_t>(nn) * K + k] : B[static_cast<size_t>(k) * N + nn];
      sa[kk][mm] = va;
      sb[kk][mm] = vb;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r] = sa[kk][ty * 4 + r];
#pragma unroll
      for (int q = 0; q < 4; ++q) b[q] = sb[kk][tx * 4 + q];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[r][q] = fmaf(a[r], b[q], acc[r][q]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int m = m0 + ty * 4 + r;
    if (m >= M) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = n0 + tx * 4 + q;
      if (n >= N) continue;
      float* c = C + static_cast<size_t>(m) * N + n;
      *c = beta != 0.0f ? fmaf(alpha, acc[r][q], beta * *c) : alpha * acc[r][q];
    }
  }
}

}  // namespace
}  // namespace dlm

extern "C" {

int dlm_bias_add_rowvec(const void* in, const void* bias, void* out, int tokens, int C, void* stream) {
  if (tokens <= 0 || C <= 0) return DLM_OK;
  DLM_REQUIRE(in && bias && out, DLM_ERR_INVALID, "bias_add_rowvec: null pointer");
  const long long n = static_cast<long long>(tokens) * C;
  dlm::bias_rowvec_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(in), static_cast<const __half*>(bias), static_cast<__half*>(out), n, C);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_bias_add_channel(const void* in, const void* bias, void* out, int N, int C, int H, int W,
                         void* stream) {
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return DLM_OK;
  DLM_REQUIRE(in && bias && out, DLM_ERR_INVALID, "bias_add_channel: null pointer");
  const long long n = static_cast<long long>(N) * C * H * W;
  dlm::bias_channel_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(in), static_cast<const __half*>(bias), static_cast<__half*>(out), n, C,
      H * W);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_conv_bias_biasch(const void* conv, const void* conv_bias, const void* tproj, void* out, int B,
                         int Cout, int H, int W, void* stream) {
  if (B <= 0 || Cout <= 0 || H <= 0 || W <= 0) return DLM_OK;
  DLM_REQUIRE(conv && conv_bias && tproj && out, DLM_ERR_INVALID, "conv_bias_biasch: null pointer");
  const long long n = static_cast<long long>(B) * Cout * H * W;
  dlm::conv_bias_two_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(conv), static_cast<const __half*>(conv_bias),
      static_cast<const __half*>(tproj), static_cast<__half*>(out), n, Cout, H * W, 0);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_conv_bias_residual(const void* conv, const void* conv_bias, const void* residual, void* out,
                           int B, int Cout, int H, int W, void* stream) {
  if (B <= 0 || Cout <= 0 || H <= 0 || W <= 0) return DLM_OK;
  DLM_REQUIRE(conv && conv_bias && residual && out, DLM_ERR_INVALID, "conv_bias_residual: null pointer");
  const long long n = static_cast<long long>(B) * Cout * H * W;
  dlm::conv_bias_two_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(conv), static_cast<const __half*>(conv_bias),
      static_cast<const __half*>(residual), static_cast<__half*>(out), n, Cout, H * W, 1);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

static int activation(const void* in, void* out, int n, int kind, void* stream) {
  if (n <= 0) return DLM_OK;
  DLM_REQUIRE(in && out, DLM_ERR_INVALID, "activation: null pointer");
  dlm::activation_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(in), static_cast<__half*>(out), n, kind);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_silu(const void* in, void* out, int n, void* stream) { return activation(in, out, n, 0, stream); }
int dlm_gelu(const void* in, void* out, int n, void* stream) { return activation(in, out, n, 1, stream); }
int dlm_gelu_tanh(const void* in, void* out, int n, void* stream) { return activation(in, out, n, 2, stream); }

int dlm_add(const void* a, const void* b, void* out, int n, void* stream) {
  if (n <= 0) return DLM_OK;
  DLM_REQUIRE(a && b && out, DLM_ERR_INVALID, "add: null pointer");
  dlm::add_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<__half*>(out), n);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_upsample_nearest2x(const void* in, void* out, int N, int C, int H, int W, void* stream) {
  if (N <= 0 || C <= 0 || H <= 0 || W <= 0) return DLM_OK;
  DLM_REQUIRE(in && out, DLM_ERR_INVALID, "upsample_nearest2x: null pointer");
  const long long n_out = static_cast<long long>(N) * C * 4 * H * W;
  dlm::upsample_nchw_kernel<<<dlm::blocks_for(n_out), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(in), static_cast<__half*>(out), n_out, H, W);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_geglu(const void* in, void* out, int tokens, int d, void* stream) {
  if (tokens <= 0 || d <= 0) return DLM_OK;
  DLM_REQUIRE(in && out, DLM_ERR_INVALID, "geglu: null pointer");
  const long long n = static_cast<long long>(tokens) * d;
  dlm::geglu_kernel<<<dlm::blocks_for(n), dlm::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(in), static_cast<__half*>(out), n, d);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_timestep_embedding(void* out, float timestep, int dim, float max_period, void* stream) {
  const int half = dim / 2;
  if (half <= 0) return DLM_OK;
  DLM_REQUIRE(out && max_period > 0.0f, DLM_ERR_INVALID, "timestep_embedding: bad argument");
  dlm::timestep_embedding_kernel<<<(half + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(out), timestep, half, logf(max_period));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K, float alpha, float beta,
                 int transA, int transB, void* stream) {
  if (M <= 0 || N <= 0) return DLM_OK;
  DLM_REQUIRE(A && B && C && K >= 0, DLM_ERR_INVALID, "gemm_f32: bad argument");
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  DLM_REQUIRE(grid.y <= 65535, DLM_ERR_INVALID, "gemm_f32: M %d too large", M);
  dlm::gemm_f32_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(A, B, C, M, N, K, alpha, beta,
                                                                          transA, transB);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

}  // extern "C"
