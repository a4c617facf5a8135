// GroupNorm and LayerNorm on NHWC / token-major fp16 activations (HBM-bound).
//
// GroupNorm (replaces launch_group_norm / _mb / _silu, reference src/kernels/groupnorm.cuh:51-108,
// groupnorm.cu:246-467) is two launches:
//   gn_stats   grid (chunks, N): each block reduces a chunk of pixels to per-group partial
//              (sum, sum of squares) in fp32, in a fixed order (deterministic, like the
//              reference's multi-block GN, groupnorm.cu:246-327);
//   gn_apply   each block first folds its image's partials (fixed order, fp64) into mean / rstd
//              per group, then writes y = (x - mean) * rstd * gamma + beta (optional SiLU) as fp16.
// The input may be the channel concatenation of two NHWC sources (the UNet up-path skip concat,
// unet.cu:250 k_concat_chw): gn_apply writes the normalised concat in one pass, so the concat
// copy never exists.
// LayerNorm (launch_layer_norm, layernorm.cuh:51-57): one warp per token row, two-pass mean /
// variance in registers.
#include <cuda_fp16.h>

#include "norm.h"
#include "ptx.cuh"

namespace dlm {

namespace {

constexpr int kGroups = 32;
constexpr int kStatThreads = 256;

__device__ __forceinline__ void load8(const __half* p, float* f) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void load8(const float* p, float* f) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x;
  f[1] = a.y;
  f[2] = a.z;
  f[3] = a.w;
  f[4] = b.x;
  f[5] = b.y;
  f[6] = b.z;
  f[7] = b.w;
}

constexpr int kStatUnroll = 8;   // independent pixel loads in flight per thread (stats)
constexpr int kApplyUnroll = 2;  // independent 16-byte loads in flight per thread (apply)
constexpr int kFoldSets = kStatThreads / kGroups;
constexpr int kBlocksPerSm = 4;  // stats / apply blocks per SM (16 warps each way would leave
                                 // the passes latency bound)

// Statistics pass.  Block (chunk, n) reduces pixels [chunk * pix_per_chunk, ...) of image n to
// per-group (sum, sum of squares) in fp32 and writes partials[(n * chunks + chunk) * 32 + g].
// The block that finishes last for image n (arrival counter, counters[n]) folds that image's
// partials in a fixed order in fp64, writes mean_rstd[n * 32 + g] = (mean, rstd) and resets the
// counter to zero for the next launch.  The fold order does not depend on which block is last,
// so the result is deterministic.  T = __half or float (fp32 input: the VAE's fp32 carries).
template <typename T>
__global__ void __launch_bounds__(kStatThreads, kBlocksPerSm)
    gn_stats_kernel(const T* __restrict__ x1, int C1, const T* __restrict__ x2, int C2,
                    int HW, int pix_per_chunk, float2* __restrict__ partials,
                    float2* __restrict__ mean_rstd, unsigned* __restrict__ counters, float eps) {
  extern __shared__ float sh[];  // [PL][C] sums then [PL][C] sumsq
  __shared__ double s_fold[2][kFoldSets][kGroups];
  __shared__ int s_last;
  griddep_wait();  // dependents launch when this grid exits
  const int C = C1 + C2;
  const int nvec = C >> 3;
  const int chunk = blockIdx.x, n = blockIdx.y, chunks = gridDim.x;
  const int PL = nvec >= kStatThreads ? 1 : kStatThreads / nvec;
  float* s_sum = sh;
  float* s_sq = sh + PL * C;
  const int p0 = chunk * pix_per_chunk;
  const int p1 = min(HW, p0 + pix_per_chunk);
  for (int t = threadIdx.x; t < PL * nvec; t += blockDim.x) {
    const int cv = t % nvec, pl = t / nvec;
    const int c = cv * 8;
    const T* base = c < C1 ? x1 + c : x2 + (c - C1);
    const int ld = c < C1 ? C1 : C2;
    float a[8], q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = q[i] = 0.0f;
    const size_t img = static_cast<size_t>(n) * HW;
    int pix = p0 + pl;
    // full groups of kStatUnroll pixels: all loads issued before the first use
    // fp32 rows are twice the bytes: half the pixels in flight keep the same bytes per thread
    constexpr int U = sizeof(T) == 4 ? kStatUnroll / 2 : kStatUnroll;
    for (; pix + (U - 1) * PL < p1; pix += U * PL) {
      float f[U][8];
#pragma unroll
      for (int u = 0; u < U; ++u) load8(base + (img + pix + u * PL) * ld, f[u]);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          a[i] += f[u][i];
          q[i] = fmaf(f[u][i], f[u][i], q[i]);
        }
    }
    for (; pix < p1; pix += PL) {
      float f[8];
      load8(base + (img + pix) * ld, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a[i] += f[i];
        q[i] = fmaf(f[i], f[i], q[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s_sum[pl * C + c + i] = a[i];
      s_sq[pl * C + c + i] = q[i];
    }
  }
  __syncthreads();
  if (threadIdx.x < kGroups) {
    const int g = threadIdx.x;
    const int cpg = C / kGroups;
    float a = 0.0f, q = 0.0f;
    for (int pl = 0; pl < PL; ++pl)
      for (int c = g * cpg; c < (g + 1) * cpg; ++c) {
        a += s_sum[pl * C + c];
        q += s_sq[pl * C + c];
      }
    partials[(static_cast<size_t>(n) * chunks + chunk) * kGroups + g] = make_float2(a, q);
  }
  // publish this block's partials, then count it in
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[n], 1u) == static_cast<unsigned>(chunks - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  {
    const int g = threadIdx.x % kGroups, set = threadIdx.x / kGroups;
    double a = 0.0, q = 0.0;
    const float2* pp = partials + static_cast<size_t>(n) * chunks * kGroups + g;
#pragma unroll 16
    for (int k = set; k < chunks; k += kFoldSets) {
      const float2 v = __ldcg(pp + static_cast<size_t>(k) * kGroups);
      a += v.x;
      q += v.y;
    }
    s_fold[0][set][g] = a;
    s_fold[1][set][g] = q;
  }
  __syncthreads();
  if (threadIdx.x < kGroups) {
    const int g = threadIdx.x;
    double a = 0.0, q = 0.0;
    for (int k = 0; k < kFoldSets; ++k) {
      a += s_fold[0][k][g];
      q += s_fold[1][k][g];
    }
    const double cnt = static_cast<double>(HW) * (C / kGroups);
    const double mean = a / cnt;
    double var = q / cnt - mean * mean;
    if (var < 0.0) var = 0.0;
    mean_rstd[n * kGroups + g] =
        make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + static_cast<double>(eps))));
    if (g == 0) counters[n] = 0u;
  }
}

// Apply pass: block (b, n) writes pixels [b * pix_per_block, ...) of image n as
// y = (x - mean) * rstd * gamma + beta (optional SiLU), fp16.  Each thread owns one 8-channel
// vector (its per-channel scale rstd * gamma and shift beta - mean * rstd * gamma stay in
// registers) and walks the block's pixels with stride PL = 256 / (C / 8).
template <typename T>
__global__ void __launch_bounds__(256, kBlocksPerSm)
    gn_apply_kernel(const T* __restrict__ x1, int C1, const T* __restrict__ x2, int C2,
                    int HW, const float2* __restrict__ mean_rstd, const __half* __restrict__ gamma,
                    const __half* __restrict__ beta, int silu, int pix_per_block,
                    __half* __restrict__ out) {
  // The image's 32 (mean, rstd) pairs once per block: read per thread, every thread of the grid
  // asks the same 256 bytes of L2 eight times and the slice holding them serialises the pass.
  __shared__ float2 s_mr[kGroups];
  griddep_wait();  // dependents launch when this grid exits
  const int C = C1 + C2;
  const int n = blockIdx.y;
  if (threadIdx.x < kGroups) s_mr[threadIdx.x] = __ldg(mean_rstd + n * kGroups + threadIdx.x);
  __syncthreads();
  const int nvec = C >> 3;
  const int cpg = C / kGroups;
  const int PL = nvec >= static_cast<int>(blockDim.x) ? 1 : blockDim.x / nvec;
  const int p0 = blockIdx.x * pix_per_block;
  const int p1 = min(HW, p0 + pix_per_block);
  const size_t img = static_cast<size_t>(n) * HW;
  for (int w = threadIdx.x; w < PL * nvec; w += blockDim.x) {
    const int cv = w % nvec, pl = w / nvec;
    const int c = cv * 8;
    float sc[8], sh[8];
    {
      float gm[8], bt[8];
      load8(gamma + c, gm);
      load8(beta + c, bt);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 mr = s_mr[(c + i) / cpg];
        sc[i] = mr.y * gm[i];
        sh[i] = bt[i] - mr.x * sc[i];
      }
    }
    const T* src = c < C1 ? x1 + c : x2 + (c - C1);
    const int ld = c < C1 ? C1 : C2;
    __half* dst = out + c;
    auto emit = [&](int pix, const float* f) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        float y0 = fmaf(f[i], sc[i], sh[i]);
        float y1 = fmaf(f[i + 1], sc[i + 1], sh[i + 1]);
        if (silu) {
          y0 = silu_f(y0);
          y1 = silu_f(y1);
        }
        o[i >> 1] = pack_half2(y0, y1);
      }
      *reinterpret_cast<uint4*>(dst + (img + pix) * C) = make_uint4(o[0], o[1], o[2], o[3]);
    };
    int pix = p0 + pl;
    // full groups of kApplyUnroll pixels: all loads issued before the first use
    for (; pix + (kApplyUnroll - 1) * PL < p1; pix += kApplyUnroll * PL) {
      float f[kApplyUnroll][8];
#pragma unroll
      for (int u = 0; u < kApplyUnroll; ++u) load8(src + (img + pix + u * PL) * ld, f[u]);
#pragma unroll
      for (int u = 0; u < kApplyUnroll; ++u) emit(pix + u * PL, f[u]);
    }
    for (; pix < p1; pix += PL) {
      float f[8];
      load8(src + (img + pix) * ld, f);
      emit(pix, f);
    }
  }
}

// One warp per row; C % 256 == 0 is not required, C % 8 == 0 and C <= 8 * 32 * kLnVec.
constexpr int kLnVec = 8;  // up to 2048 channels
__global__ void __launch_bounds__(256)
    layer_norm_kernel(const __half* __restrict__ x, const __half* __restrict__ gamma,
                      const __half* __restrict__ beta, __half* __restrict__ out, int rows, int C,
                      float eps) {
  griddep_wait();  // dependents launch when this grid exits
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int nvec = C >> 3;
  const __half* xr = x + static_cast<size_t>(warp) * C;
  float v[kLnVec][8];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kLnVec; ++k) {
    const int cv = lane + 32 * k;
    if (cv < nvec) {
      load8(xr + cv * 8, v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[k][i];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / C;
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < kLnVec; ++k) {
    const int cv = lane + 32 * k;
    if (cv < nvec) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[k][i] - mean;
        q = fmaf(d, d, q);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / C + eps);
  __half* orow = out + static_cast<size_t>(warp) * C;
#pragma unroll
  for (int k = 0; k < kLnVec; ++k) {
    const int cv = lane + 32 * k;
    if (cv < nvec) {
      float gm[8], bt[8];
      if (gamma) load8(gamma + cv * 8, gm);
      if (beta) load8(beta + cv * 8, bt);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        float y0 = (v[k][i] - mean) * rstd, y1 = (v[k][i + 1] - mean) * rstd;
        if (gamma) {
          y0 *= gm[i];
          y1 *= gm[i + 1];
        }
        if (beta) {
          y0 += bt[i];
          y1 += bt[i + 1];
        }
        o[i >> 1] = pack_half2(y0, y1);
      }
      *reinterpret_cast<uint4*>(orow + cv * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace

// Scratch layout (float2 units): [N * 32 (mean, rstd)] [counters: N unsigned, padded to 32 float2]
// [partials: N * chunks * 32].  The fixed-size head does not depend on the SM count.
size_t gn_head_elems(int N) { return static_cast<size_t>(N) * kGroups + ((N + 63) / 64) * 32; }

int gn_chunks(int N, int HW, int sms, int* ppc_out) {
  int chunks = (kBlocksPerSm * sms + N - 1) / N;
  int ppc = (HW + chunks - 1) / chunks;
  if (ppc < 8) ppc = 8;
  *ppc_out = ppc;
  return (HW + ppc - 1) / ppc;
}

int gn_plan(GnOp* op, const __half* x1, int C1, const __half* x2, int C2, int N, int HW,
            const __half* gamma, const __half* beta, float eps, bool silu, __half* out,
            float2* partials, size_t partial_cap) {
  const int C = C1 + C2;
  DLM_REQUIRE(op && x1 && gamma && beta && out && partials, DLM_ERR_INVALID, "gn: null pointer");
  DLM_REQUIRE(C % kGroups == 0 && C1 % 8 == 0 && C2 % 8 == 0 && (C2 == 0 || x2 != nullptr),
              DLM_ERR_INVALID, "gn: channels %d+%d must be multiples of 8 and of 32 in total", C1, C2);
  DLM_REQUIRE(C <= 4096, DLM_ERR_INVALID, "gn: at most 4096 channels");
  DLM_REQUIRE(N > 0 && HW > 0 && N <= 65535, DLM_ERR_INVALID, "gn: bad batch %d / pixels %d", N, HW);
  const int sms = num_sms();
  int ppc = 0;
  const int chunks = gn_chunks(N, HW, sms, &ppc);
  const size_t need = gn_head_elems(N) + static_cast<size_t>(N) * chunks * kGroups;
  DLM_REQUIRE(need <= partial_cap, DLM_ERR_NOMEM, "gn: partial buffer too small (%zu < %zu)",
              partial_cap, need);
  op->x1 = x1;
  op->x2 = x2;
  op->C1 = C1;
  op->C2 = C2;
  op->N = N;
  op->HW = HW;
  op->gamma = gamma;
  op->beta = beta;
  op->eps = eps;
  op->silu = silu;
  op->out = out;
  op->mean_rstd = partials;
  op->counters = reinterpret_cast<unsigned*>(partials + static_cast<size_t>(N) * kGroups);
  op->partials = partials + gn_head_elems(N);
  op->chunks = chunks;
  op->pix_per_chunk = ppc;
  const int nvec = C / 8;
  const int PL = nvec >= kStatThreads ? 1 : kStatThreads / nvec;
  op->stat_smem = 2 * PL * C * static_cast<int>(sizeof(float));
  const int per_img = (kBlocksPerSm * sms + N - 1) / N;
  int ppb = (HW + per_img - 1) / per_img;
  if (ppb < 4) ppb = 4;
  op->pix_per_block = ppb;
  return DLM_OK;
}

int gn_plan_f32(GnOp* op, const float* x, int C, int N, int HW, const __half* gamma,
                const __half* beta, float eps, bool silu, __half* out, float2* partials,
                size_t partial_cap) {
  DLM_REQUIRE(x != nullptr, DLM_ERR_INVALID, "gn: null input");
  // plan as a single-source fp16 problem of the same geometry, then read fp32
  int rc = gn_plan(op, reinterpret_cast<const __half*>(x), C, nullptr, 0, N, HW, gamma, beta, eps,
                   silu, out, partials, partial_cap);
  if (rc != DLM_OK) return rc;
  op->xf = x;
  op->x1 = nullptr;
  return DLM_OK;
}

size_t gn_partial_elems(int N, int HW) {
  const int sms = 148 * 2;  // generous bound for any SM count up to 296
  int ppc = 0;
  const int chunks = gn_chunks(N, HW > 0 ? HW : 1, sms, &ppc);
  const int chunks_any = (kBlocksPerSm * sms + N - 1) / N;  // upper bound for any HW
  return gn_head_elems(N) + static_cast<size_t>(N) * (chunks > chunks_any ? chunks : chunks_any) * kGroups;
}

size_t gn_counter_bytes(int N) { return static_cast<size_t>(N) * sizeof(unsigned); }

int gn_launch(const GnOp& op, cudaStream_t s) {
  // stat_smem <= 2 * 256 * 8 floats * 4 B (PL * C <= 256 * 8 for C / 8 < 256) or 2 * C * 4 B
  // (C <= 4096): within the 48 KB default together with the 4 KB fold buffer.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.chunks, op.N, 1);
  cfg.blockDim = dim3(kStatThreads, 1, 1);
  cfg.dynamicSmemBytes = op.stat_smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  if (op.xf) {
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gn_stats_kernel<float>, op.xf, op.C1,
                                      static_cast<const float*>(nullptr), 0, op.HW,
                                      op.pix_per_chunk, op.partials, op.mean_rstd, op.counters,
                                      op.eps));
  } else {
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gn_stats_kernel<__half>, op.x1, op.C1, op.x2, op.C2,
                                      op.HW, op.pix_per_chunk, op.partials, op.mean_rstd,
                                      op.counters, op.eps));
  }
  const int blocks = (op.HW + op.pix_per_block - 1) / op.pix_per_block;
  cfg.gridDim = dim3(blocks, op.N, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  if (op.xf) {
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gn_apply_kernel<float>, op.xf, op.C1,
                                      static_cast<const float*>(nullptr), 0, op.HW,
                                      static_cast<const float2*>(op.mean_rstd), op.gamma, op.beta,
                                      op.silu ? 1 : 0, op.pix_per_block, op.out));
  } else {
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, gn_apply_kernel<__half>, op.x1, op.C1, op.x2, op.C2,
                                      op.HW, static_cast<const float2*>(op.mean_rstd), op.gamma,
                                      op.beta, op.silu ? 1 : 0, op.pix_per_block, op.out));
  }
  return DLM_OK;
}

int layer_norm(const __half* x, const __half* gamma, const __half* beta, __half* out, int rows, int C,
               float eps, cudaStream_t s) {
  DLM_REQUIRE(x && out, DLM_ERR_INVALID, "layer_norm: null pointer");
  DLM_REQUIRE(C % 8 == 0 && C <= 8 * 32 * kLnVec, DLM_ERR_INVALID,
              "layer_norm: C=%d must be a multiple of 8 and <= %d", C, 8 * 32 * kLnVec);
  const int warps_per_block = 8;
  const int blocks = (rows + warps_per_block - 1) / warps_per_block;
  layer_norm_kernel<<<blocks, warps_per_block * 32, 0, s>>>(x, gamma, beta, out, rows, C, eps);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

}  // namespace dlm

extern "C" {

size_t dlm_group_norm_nhwc_scratch_bytes(int N, int HW) {
  return dlm::gn_partial_elems(N, HW) * sizeof(float2);
}

int dlm_group_norm_nhwc(const void* x1, int C1, const void* x2, int C2, int N, int HW,
                        const void* gamma, const void* beta, float eps, int groups, int silu,
                        void* out, void* scratch, size_t scratch_bytes, void* stream) {
  if (N == 0 || HW == 0 || C1 + C2 == 0) return DLM_OK;
  DLM_REQUIRE(groups == 32, DLM_ERR_UNSUPPORTED, "group_norm_nhwc: groups must be 32");
  DLM_REQUIRE(scratch != nullptr, DLM_ERR_INVALID, "group_norm_nhwc: null scratch");
  dlm::GnOp op;
  int rc = dlm::gn_plan(&op, static_cast<const __half*>(x1), C1, static_cast<const __half*>(x2), C2,
                        N, HW, static_cast<const __half*>(gamma), static_cast<const __half*>(beta),
                        eps, silu != 0, static_cast<__half*>(out), static_cast<float2*>(scratch),
                        scratch_bytes / sizeof(float2));
  if (rc != DLM_OK) return rc;
  // the caller's scratch may hold anything: start the arrival counters at zero
  DLM_CHECK_CUDA(cudaMemsetAsync(op.counters, 0, dlm::gn_counter_bytes(N),
                                 static_cast<cudaStream_t>(stream)));
  return dlm::gn_launch(op, static_cast<cudaStream_t>(stream));
}

int dlm_launch_layer_norm(const void* in, const void* gamma, const void* beta, void* out, int rows,
                          int C, float eps, void* stream) {
  if (rows == 0 || C == 0) return DLM_OK;
  return dlm::layer_norm(static_cast<const __half*>(in), static_cast<const __half*>(gamma),
                         static_cast<const __half*>(beta), static_cast<__half*>(out), rows, C, eps,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
