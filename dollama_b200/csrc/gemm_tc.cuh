// tcgen05 GEMM for sm_100a: C[M, N] = epi(A[M, K] * B[N, K]^T), fp16 operands, fp32
// accumulation in tensor memory.
//
// One persistent CTA per SM walks output tiles of 128 x BN.  Roles (192 threads):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of
//               two TMEM accumulators (2 x BN fp32 columns) and commits to the barriers;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (each warp owns the 32 TMEM lanes of
//               its quadrant, warp % 4), fused bias / per-image bias / SiLU / GEGLU / residual,
//               fp16 store; the second accumulator lets tile i's epilogue overlap tile i+1's MMAs.
//
// The A operand is either a dense row-major matrix (2D tensor map) or an implicit-GEMM view of
// an NHWC activation for a 3x3 / 1x1 convolution: each 64-wide k-block is one (tap, 64-channel)
// slice, fetched as a 4D TMA box {64 ch, bw, bh, 1} whose out-of-range coordinates are filled
// with zeros by the TMA unit — that IS the conv's zero padding.  A stride-2 3x3 conv reads a
// 5D view of the four (row, col) parity planes of its input.  No im2col buffer exists.
//
// No load uses cluster multicast: every CTA fetches its own tiles.
#pragma once

#include "../../include/dollama_b200.h"
#include "ptx.cuh"

namespace dlm {

// One K segment of an implicit-GEMM convolution.
struct ConvSeg {
  int map;      // A tensor map index (0..2)
  int kind;     // 0: 3x3 stride 1 (4D map), 1: 1x1 centre tap (4D map),
                // 2: 3x3 stride 2 from parity planes (5D map)
  int cblocks;  // number of 64-channel blocks
};

struct GemmParams {
  int M, N;           // output rows; GEMM N (output has N/2 columns with GEGLU)
  int num_kb;         // k-blocks of 64
  int m_tiles, n_tiles;
  int amode;          // 0: dense A, 1: implicit conv
  int oH, oW, bh, bw; // conv output geometry and per-tile pixel box (bh * bw == 128)
  int nseg;
  ConvSeg seg[3];
  unsigned flags;     // DLM_EPI_* bits
  float alpha;        // scale of the accumulator
  float resid_scale;  // scale of the residual term
  __half* out;
  int ldo;
  const __half* bias;
  const __half* bias2d;
  int rows_per_img;
  int ldb2;  // row stride of bias2d
  const __half* resid;
  int ldr;
  int* status;
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;

__host__ __device__ constexpr int gemm_stage_bytes(int BN) { return (kGemmBM + BN) * kGemmBK * 2; }
__host__ __device__ constexpr int gemm_stages(int BN) {
  return ((225 * 1024 - 2048) / gemm_stage_bytes(BN)) > 8 ? 8
                                                            : ((225 * 1024 - 2048) / gemm_stage_bytes(BN));
}
__host__ __device__ constexpr int gemm_smem_bytes(int BN) {
  return gemm_stages(BN) * gemm_stage_bytes(BN) + 1024 + 256;
}
__host__ __device__ constexpr uint32_t gemm_tmem_cols(int BN) {
  return (2 * BN) <= 32 ? 32 : (2 * BN) <= 64 ? 64 : (2 * BN) <= 128 ? 128 : (2 * BN) <= 256 ? 256 : 512;
}

__device__ __forceinline__ void load_half8(const __half* p, float* f) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void load_half8_nc(const __half* p, float* f) {
  // residual may alias the output: plain (coherent) load
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  constexpr int A_BYTES = kGemmBM * kGemmBK * 2;
  constexpr int B_BYTES = BN * kGemmBK * 2;
  constexpr int STAGES = gemm_stages(BN);
  constexpr uint32_t TMEM_COLS = gemm_tmem_cols(BN);
  static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "UMMA N for M=128");
  static_assert(2 * BN <= 512, "two accumulators must fit TMEM");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA0);
    if (p.amode == 1) {
      tma_prefetch_desc(&tmA1);
      tma_prefetch_desc(&tmA2);
    }
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  const int num_tiles = p.m_tiles * p.n_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.n_tiles) * kGemmBM;
        const int n0 = (t % p.n_tiles) * BN;
        if (p.amode == 0) {
          for (int kb = 0; kb < p.num_kb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tmA0, &full[stage], kb * kGemmBK, m0);
            tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * kGemmBK, n0);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        } else {
          const int hw = p.oH * p.oW;
          const int img = m0 / hw;
          const int rem = m0 - img * hw;
          const int oh0 = rem / p.oW;
          const int ow0 = rem - oh0 * p.oW;
          int kb = 0;
          for (int s = 0; s < p.nseg && ok; ++s) {
            const ConvSeg sg = p.seg[s];
            const CUtensorMap* am = sg.map == 0 ? &tmA0 : (sg.map == 1 ? &tmA1 : &tmA2);
            const int ntaps = sg.kind == 1 ? 1 : 9;
            for (int tap = 0; tap < ntaps && ok; ++tap) {
              const int kh = tap / 3, kw = tap - (tap / 3) * 3;
              for (int cb = 0; cb < sg.cblocks; ++cb) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
                  ok = false;
                  break;
                }
                mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
                uint8_t* dstA = sA + stage * A_BYTES;
                if (sg.kind == 0) {
                  tma_load_4d(dstA, am, &full[stage], cb * 64, ow0 + kw - 1, oh0 + kh - 1, img);
                } else if (sg.kind == 1) {
                  tma_load_4d(dstA, am, &full[stage], cb * 64, ow0, oh0, img);
                } else {
                  // input row 2*oh + kh - 1: kh=0 -> odd plane, row oh-1; kh=1 -> even, oh;
                  // kh=2 -> odd, oh.  Same for columns.
                  const int pr = (kh == 1) ? 0 : 1, dr = (kh == 0) ? -1 : 0;
                  const int pc = (kw == 1) ? 0 : 1, dc = (kw == 0) ? -1 : 0;
                  tma_load_5d(dstA, am, &full[stage], cb * 64, ow0 + dc, oh0 + dr, img, pr * 2 + pc);
                }
                tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * kGemmBK, n0);
                ++kb;
                if (++stage == STAGES) {
                  stage = 0;
                  phase ^= 1;
                }
              }
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kGemmBM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tbase + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t ad = sw128_desc(a_base + k * 32, 16, 1024);
            const uint64_t bd = sw128_desc(b_base + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quad = warp & 3;
    const int out_cols = (p.flags & DLM_EPI_GEGLU) ? (p.N >> 1) : p.N;
    (void)out_cols;
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int m0 = (t / p.n_tiles) * kGemmBM;
      const int n0 = (t % p.n_tiles) * BN;
      const int row = m0 + quad * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tbase + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= p.N) break;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c, r);
        tmem_ld_wait();
        if (!row_ok) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
        const int n = n0 + c;
        if (p.flags & DLM_EPI_BIAS) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float b[8];
            load_half8(p.bias + n + j, b);
#pragma unroll
            for (int q = 0; q < 8; ++q) v[j + q] += b[q];
          }
        }
        if (p.flags & DLM_EPI_BIAS2D) {
          const __half* b2 = p.bias2d + static_cast<size_t>(row / p.rows_per_img) * p.ldb2 + n;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float b[8];
            load_half8(b2 + j, b);
#pragma unroll
            for (int q = 0; q < 8; ++q) v[j + q] += b[q];
          }
        }
        if (p.flags & DLM_EPI_SILU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
        }
        if (p.flags & DLM_EPI_GEGLU) {
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float a0 = v[4 * j] * gelu_erf_f(v[4 * j + 1]);
            const float a1 = v[4 * j + 2] * gelu_erf_f(v[4 * j + 3]);
            o[j] = pack_half2(a0, a1);
          }
          uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<size_t>(row) * p.ldo + (n >> 1));
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else {
          if (p.flags & DLM_EPI_RESID) {
            const __half* rs = p.resid + static_cast<size_t>(row) * p.ldr + n;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              float b[8];
              load_half8_nc(rs + j, b);
#pragma unroll
              for (int q = 0; q < 8; ++q) v[j + q] += p.resid_scale * b[q];
            }
          }
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = pack_half2(v[2 * j], v[2 * j + 1]);
          uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<size_t>(row) * p.ldo + n);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
          dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

}  // namespace dlm
