// The reference kernel library's remaining NCHW host entries, for callers outside this library's
// NHWC model graphs (the UNet / VAE handles never call these):
//
//   dlm_group_norm_nchw            src/kernels/groupnorm.cuh:51-108 launch_group_norm /
//                                  launch_group_norm_mb / launch_group_norm_silu: GroupNorm over
//                                  NCHW fp16 (in place allowed), optional SiLU after an fp16
//                                  rounding of the normalised value (the reference's silu variant
//                                  rounds the GroupNorm result first, groupnorm.cuh:92-99)
//   dlm_conv2d_direct_nchw         src/kernels/conv2d.cuh:65-69 launch_conv2d_direct and, with
//                                  fp32 activations, :79-82 launch_conv2d_f32_gemm: any kernel
//                                  size / stride / padding / dilation, fp32 accumulation, bias
//                                  folded into the accumulator, one rounding at the store
//   dlm_conv2d_uses_gemm_bias_path src/kernels/conv2d.cuh:54-56: whether a convolution of this
//                                  shape runs on the implicit-GEMM tensor-core path
//                                  (dlm_conv2d_nhwc), which rounds the bias-free convolution once
//                                  to fp16 — so a caller may pass bias = NULL and add the bias in
//                                  a later pass with the reference's two-rounding sequence; other
//                                  shapes take the direct convolution
//
// GroupNorm numerics: each (image, group) is one contiguous range of (C / groups) * HW values.
// Blocks reduce slices of it to (sum, sum of squares) in fp32 around a shift (the group's first
// value, which all its blocks read) so that a large mean does not cancel the variance; the last
// block of a group (arrival counter) folds its slices in fixed order in fp64 into (mean, rstd).
// The result does not depend on launch timing: the fold order is the slice order.
#include <cuda_fp16.h>

#include "common.h"

namespace dlm {
namespace {

constexpr int kGnThreads = 256;
constexpr int kGnMaxSlices = 32;   // slices per (image, group)
constexpr int kGnMinSlice = 2048;  // values per slice at least

struct GnGeom {
  int N, C, HW, groups;
  long long per_group;  // (C / groups) * HW
  int slices;
  long long slice_len;
};

GnGeom gn_geom(int N, int C, int HW, int groups, int sms) {
  GnGeom g{N, C, HW, groups, static_cast<long long>(C / groups) * HW, 1, 0};
  const long long target = 4LL * sms;
  long long s = (target + static_cast<long long>(N) * groups - 1) / (static_cast<long long>(N) * groups);
  const long long by_len = (g.per_group + kGnMinSlice - 1) / kGnMinSlice;
  if (s > by_len) s = by_len;
  if (s > kGnMaxSlices) s = kGnMaxSlices;
  if (s < 1) s = 1;
  g.slice_len = (g.per_group + s - 1) / s;
  g.slices = static_cast<int>((g.per_group + g.slice_len - 1) / g.slice_len);
  return g;
}

size_t gn_nchw_head_bytes(int N, int groups) {
  const size_t ng = static_cast<size_t>(N) * groups;
  return ((ng * sizeof(float2) + 255) / 256) * 256 + ((ng * sizeof(unsigned) + 255) / 256) * 256;
}

// grid (slices, N * groups)
__global__ void __launch_bounds__(kGnThreads)
gn_nchw_stats_kernel(const __half* __restrict__ x, long long per_group, long long slice_len,
                     int slices, float2* __restrict__ partials, float2* __restrict__ mean_rstd,
                     unsigned* __restrict__ counters, float eps) {
  const int ng = blockIdx.y;
  const __half* base = x + static_cast<long long>(ng) * per_group;
  const float shift = __half2float(base[0]);
  const long long lo = static_cast<long long>(blockIdx.x) * slice_len;
  long long hi = lo + slice_len;
  if (hi > per_group) hi = per_group;
  float s1 = 0.0f, s2 = 0.0f;
  for (long long i = lo + threadIdx.x; i < hi; i += kGnThreads) {
    const float d = __half2float(base[i]) - shift;
    s1 += d;
    s2 = fmaf(d, d, s2);
  }
  __shared__ float r1[kGnThreads / 32], r2[kGnThreads / 32];
  __shared__ bool s_last;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    r1[warp] = s1;
    r2[warp] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.0f, b = 0.0f;
    for (int w = 0; w < kGnThreads / 32; ++w) {
      a += r1[w];
      b += r2[w];
    }
    partials[static_cast<long long>(ng) * slices + blockIdx.x] = make_float2(a, b);
    __threadfence();
    s_last = atomicAdd(&counters[ng], 1u) == static_cast<unsigned>(slices - 1);
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  double a = 0.0, b = 0.0;
  const volatile float2* p = partials + static_cast<long long>(ng) * slices;
  for (int k = 0; k < slices; ++k) {
    a += static_cast<double>(p[k].x);
    b += static_cast<double>(p[k].y);
  }
  const double n = static_cast<double>(per_group);
  const double m = a / n;
  double var = b / n - m * m;
  if (var < 0.0) var = 0.0;
  mean_rstd[ng] = make_float2(static_cast<float>(m + shift),
                              static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps))));
  counters[ng] = 0u;
}

__device__ __forceinline__ float gn_out(float v, float2 mr, float ga, float be, bool silu) {
  float y = (v - mr.x) * mr.y * ga + be;
  if (silu) {
    y = __half2float(__float2half(y));
    y = y / (1.0f + __expf(-y));
  }
  return y;
}

__global__ void __launch_bounds__(kGnThreads)
gn_nchw_apply_kernel(const __half* x, const __half* __restrict__ gamma,
                     const __half* __restrict__ beta, __half* y, int C, int HW, int cpg,
                     long long total, const float2* __restrict__ mean_rstd, int silu) {
  for (long long i = blockIdx.x * static_cast<long long>(kGnThreads) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * kGnThreads) {
    const long long nc = i / HW;
    const int c = static_cast<int>(nc % C);
    const long long n = nc / C;
    const float2 mr = mean_rstd[n * (C / cpg) + c / cpg];
    y[i] = __float2half(gn_out(__half2float(x[i]), mr, __half2float(gamma[c]),
                               __half2float(beta[c]), silu != 0));
  }
}

// Direct convolution: one thread per output value, NCHW, fp32 accumulation.
template <typename Tin, typename Tout>
__global__ void conv_direct_kernel(const Tin* __restrict__ in, const __half* __restrict__ w,
                                   const __half* __restrict__ bias, Tout* __restrict__ out, int N,
                                   int Cin, int H, int W, int Cout, int KH, int KW, int Ho, int Wo,
                                   int sh, int sw, int ph, int pw, int dh, int dw) {
  const long long total = static_cast<long long>(N) * Cout * Ho * Wo;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int wo = static_cast<int>(i % Wo);
    const int ho = static_cast<int>((i / Wo) % Ho);
    const int co = static_cast<int>((i / (static_cast<long long>(Wo) * Ho)) % Cout);
    const int n = static_cast<int>(i / (static_cast<long long>(Wo) * Ho * Cout));
    float acc = bias ? __half2float(bias[co]) : 0.0f;
    for (int ci = 0; ci < Cin; ++ci) {
      const Tin* ip = in + (static_cast<long long>(n) * Cin + ci) * H * W;
      const __half* wp = w + (static_cast<long long>(co) * Cin + ci) * KH * KW;
      for (int r = 0; r < KH; ++r) {
        const int hi = ho * sh - ph + r * dh;
        if (hi < 0 || hi >= H) continue;
        for (int s = 0; s < KW; ++s) {
          const int wi = wo * sw - pw + s * dw;
          if (wi < 0 || wi >= W) continue;
          float v;
          if constexpr (sizeof(Tin) == 2) v = __half2float(ip[static_cast<long long>(hi) * W + wi]);
          else v = ip[static_cast<long long>(hi) * W + wi];
          acc = fmaf(v, __half2float(wp[r * KW + s]), acc);
        }
      }
    }
    if constexpr (sizeof(Tout) == 2) out[i] = __float2half(acc);
    else out[i] = acc;
  }
}

inline int grid_for(long long n, int threads) {
  const long long b = (n + threads - 1) / threads;
  return static_cast<int>(b < 148LL * 64 ? b : 148LL * 64);
}

}  // namespace
}  // namespace dlm

extern "C" {

size_t dlm_group_norm_nchw_scratch_bytes(int N, int groups) {
  if (N <= 0 || groups <= 0) return 0;
  return dlm::gn_nchw_head_bytes(N, groups) +
         static_cast<size_t>(N) * groups * dlm::kGnMaxSlices * sizeof(float2);
}

int dlm_group_norm_nchw(const void* in, const void* gamma, const void* beta, void* out, int N,
                        int C, int H, int W, int groups, float eps, int silu, void* scratch,
                        size_t scratch_bytes, void* stream) {
  if (N == 0 || C == 0 || H == 0 || W == 0) return DLM_OK;
  DLM_REQUIRE(in && gamma && beta && out && scratch, DLM_ERR_INVALID, "group_norm_nchw: null pointer");
  DLM_REQUIRE(N > 0 && C > 0 && H > 0 && W > 0 && groups > 0 && C % groups == 0, DLM_ERR_INVALID,
              "group_norm_nchw: C=%d must be a positive multiple of groups=%d", C, groups);
  DLM_REQUIRE(static_cast<long long>(N) * groups <= 65535, DLM_ERR_INVALID,
              "group_norm_nchw: N * groups above 65535");
  const size_t need = dlm_group_norm_nchw_scratch_bytes(N, groups);
  DLM_REQUIRE(scratch_bytes >= need, DLM_ERR_INVALID, "group_norm_nchw: scratch %zu < %zu bytes",
              scratch_bytes, need);
  const int HW = H * W;
  const dlm::GnGeom g = dlm::gn_geom(N, C, HW, groups, dlm::num_sms());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* base = static_cast<char*>(scratch);
  const size_t ng = static_cast<size_t>(N) * groups;
  float2* mean_rstd = reinterpret_cast<float2*>(base);
  unsigned* counters = reinterpret_cast<unsigned*>(base + ((ng * sizeof(float2) + 255) / 256) * 256);
  float2* partials = reinterpret_cast<float2*>(base + dlm::gn_nchw_head_bytes(N, groups));
  DLM_CHECK_CUDA(cudaMemsetAsync(counters, 0, ng * sizeof(unsigned), s));
  dlm::gn_nchw_stats_kernel<<<dim3(g.slices, static_cast<unsigned>(ng)), dlm::kGnThreads, 0, s>>>(
      static_cast<const __half*>(in), g.per_group, g.slice_len, g.slices, partials, mean_rstd,
      counters, eps);
  DLM_CHECK_CUDA(cudaGetLastError());
  const long long total = static_cast<long long>(ng) * g.per_group;
  dlm::gn_nchw_apply_kernel<<<dlm::grid_for(total, dlm::kGnThreads), dlm::kGnThreads, 0, s>>>(
      static_cast<const __half*>(in), static_cast<const __half*>(gamma),
      static_cast<const __half*>(beta), static_cast<__half*>(out), C, HW, C / groups, total,
      mean_rstd, silu);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_conv2d_direct_nchw(const void* in, int in_f32, const void* weight, const void* bias,
                           void* out, int out_f32, int N, int Cin, int H, int W, int Cout, int KH,
                           int KW, int Hout, int Wout, int stride_h, int stride_w, int pad_h,
                           int pad_w, int dil_h, int dil_w, void* stream) {
  if (N == 0 || Cin == 0 || Cout == 0 || Hout == 0 || Wout == 0) return DLM_OK;
  DLM_REQUIRE(in && weight && out, DLM_ERR_INVALID, "conv2d_direct: null pointer");
  DLM_REQUIRE(N > 0 && Cin > 0 && H > 0 && W > 0 && Cout > 0 && KH > 0 && KW > 0 && Hout > 0 &&
                  Wout > 0 && stride_h > 0 && stride_w > 0 && pad_h >= 0 && pad_w >= 0 &&
                  dil_h > 0 && dil_w > 0,
              DLM_ERR_INVALID, "conv2d_direct: invalid dimensions");
  DLM_REQUIRE(Hout == (H + 2 * pad_h - dil_h * (KH - 1) - 1) / stride_h + 1 &&
                  Wout == (W + 2 * pad_w - dil_w * (KW - 1) - 1) / stride_w + 1,
              DLM_ERR_INVALID, "conv2d_direct: Hout / Wout do not match the geometry");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long total = static_cast<long long>(N) * Cout * Hout * Wout;
  const int grid = dlm::grid_for(total, 128);
  const __half* w = static_cast<const __half*>(weight);
  const __half* b = static_cast<const __half*>(bias);
#define DLM_CONV_DIRECT(TI, TO)                                                                 \
  dlm::conv_direct_kernel<TI, TO><<<grid, 128, 0, s>>>(                                         \
      static_cast<const TI*>(in), w, b, static_cast<TO*>(out), N, Cin, H, W, Cout, KH, KW, Hout, \
      Wout, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w)
  if (in_f32 && out_f32) DLM_CONV_DIRECT(float, float);
  else if (in_f32) DLM_CONV_DIRECT(float, __half);
  else if (out_f32) DLM_CONV_DIRECT(__half, float);
  else DLM_CONV_DIRECT(__half, __half);
#undef DLM_CONV_DIRECT
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int dlm_conv2d_uses_gemm_bias_path(int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                   int stride_h, int stride_w, int pad_h, int pad_w, int dil_h,
                                   int dil_w) {
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0) return 0;
  const bool k3 = KH == 3 && KW == 3 && pad_h == 1 && pad_w == 1 && stride_h == stride_w &&
                  (stride_h == 1 || (stride_h == 2 && H % 2 == 0 && W % 2 == 0));
  const bool k1 = KH == 1 && KW == 1 && pad_h == 0 && pad_w == 0 && stride_h == 1 && stride_w == 1;
  if (!(k3 || k1) || dil_h != 1 || dil_w != 1) return 0;
  // the implicit-GEMM convolution's granularity: 64-channel K blocks, 32-column output chunks,
  // output tiles of 128 pixels made of whole rows (or whole multiples of a row)
  const int oH = H / stride_h, oW = W / stride_w;
  const bool tiles = oW >= 128 ? (oW % 128 == 0) : (128 % oW == 0 && oH % (128 / oW) == 0);
  return (Cin % 64 == 0 && Cout % 32 == 0 && tiles) ? 1 : 0;
}

}  // extern "C"
