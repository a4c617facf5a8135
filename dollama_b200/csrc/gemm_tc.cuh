// tcgen05 GEMM for sm_100a: C[M, N] = epi(A[M, K] * B[N, K]^T), fp16 operands, fp32
// accumulation in tensor memory.
//
// One persistent CTA per SM walks output tiles of 128 x BN.  Roles (320 threads):
//   warp 0      TMA producer: streams 128x64 A and BNx64 B tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of
//               two TMEM accumulators (2 x BN fp32 columns) and commits to the barriers;
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (a warp may only read the 32 TMEM lanes
//               of its quadrant, warp % 4, so two warps share each quadrant and take alternate
//               32-column chunks), fused bias / per-image bias / SiLU / GEGLU / residual, fp16
//               store; the second accumulator lets tile i's epilogue overlap tile i+1's MMAs.
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
  // row statistics of the fp16 output (kEpiRowStats): per row and N tile, (mean, M2) of the tile's
  // stored values, at stats_out[row * stats_ld + n_tile]
  float2* stats_out;
  int stats_ld;
  // LayerNorm fold (kEpiLnFold): the A operand is the raw x whose LayerNorm the reference applies;
  // W was prescaled by gamma, and  out = rstd * (acc - mean * ln_u[n]) + ln_v[n]  with mean / rstd
  // merged from the producer's row statistics stats_in[row * stats_in_parts + i] (tiles of
  // stats_in_tile columns over ln_C columns)
  const float2* stats_in;
  int stats_in_parts, stats_in_tile, ln_C;
  float ln_eps;
  const float* ln_u;
  const float* ln_v;
  int* status;
  // stream-K (sk_ctas > 0, single-CTA kernel only): the m_tiles * n_tiles * num_kb k-block
  // iterations are split evenly over sk_ctas CTAs (the whole grid, all resident at once), so a
  // launch with fewer tiles than SMs still keeps every SM busy.  A tile cut between CTAs is
  // finished by the CTA holding its first k-block (its owner, which reaches that segment last):
  // it adds, in CTA order, the fp32 partial accumulators that the following CTAs wrote to
  // sk_ws[cta] (always their first segment) and released through sk_flags[cta], then clears those
  // flags for the next launch.
  int sk_ctas;
  float* sk_ws;   // [sk_ctas][128][BN] fp32
  int* sk_flags;  // [sk_ctas], zero between launches
};

// Internal epilogue flags (beyond the public DLM_EPI_* bits).
constexpr unsigned kEpiRowStats = 1u << 8;
constexpr unsigned kEpiLnFold = 1u << 9;
constexpr unsigned kEpiOutF32 = 1u << 10;    // output stored as fp32 (p.out points to float)
constexpr unsigned kEpiResidF32 = 1u << 11;  // residual read as fp32 (p.resid points to float)
// Kernel template argument FL: the epilogue flags fixed at compile time, so that an instantiation
// holds only its own epilogue path (the generic path's size costs instruction-cache misses on
// every chunk); kEpiDyn reads p.flags at run time instead.
constexpr unsigned kEpiDyn = 0xFFFFFFFFu;
__host__ __device__ constexpr unsigned epi_flags(unsigned FL, unsigned runtime) {
  return FL == kEpiDyn ? runtime : FL;
}

// Contiguous k-block iteration range [a, b) of CTA `cta` under stream-K.
__device__ __forceinline__ void sk_range(const GemmParams& p, int cta, long long& a, long long& b) {
  const long long total = static_cast<long long>(p.m_tiles) * p.n_tiles * p.num_kb;
  const long long q = total / p.sk_ctas, r = total % p.sk_ctas;
  a = cta * q + (cta < r ? cta : r);
  b = a + q + (cta < r ? 1 : 0);
}

// One unit of a CTA's work: k-blocks [kb0, kb1) of one output tile.
struct TileSeg {
  int tile, kb0, kb1;
};

// This CTA's work, identical in the producer, MMA and epilogue warps: whole tiles with stride
// gridDim (kb0 = 0, kb1 = num_kb), or under stream-K the tile segments of its iteration range.
struct SegIter {
  long long it, it1;
  int t;
  __device__ __forceinline__ void init(const GemmParams& p) {
    if (p.sk_ctas > 0)
      sk_range(p, blockIdx.x, it, it1);
    else
      t = blockIdx.x;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, TileSeg& sg) {
    if (p.sk_ctas > 0) {
      if (it >= it1) return false;
      sg.tile = static_cast<int>(it / p.num_kb);
      sg.kb0 = static_cast<int>(it - static_cast<long long>(sg.tile) * p.num_kb);
      const long long end = it1 - it + sg.kb0;
      sg.kb1 = end < p.num_kb ? static_cast<int>(end) : p.num_kb;
      it += sg.kb1 - sg.kb0;
      return true;
    }
    if (t >= p.m_tiles * p.n_tiles) return false;
    sg.tile = t;
    sg.kb0 = 0;
    sg.kb1 = p.num_kb;
    t += gridDim.x;
    return true;
  }
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmEpiWarps = 8;  // two per TMEM lane quadrant
constexpr int kGemmThreads = 64 + 32 * kGemmEpiWarps;

__host__ __device__ constexpr int gemm_stage_bytes(int BN) { return (kGemmBM + BN) * kGemmBK * 2; }
// Epilogue staging: each epilogue warp owns two 2 KB buffers (32 rows x 32 fp16 columns, 64-byte
// swizzled) through which its outputs leave by TMA bulk stores; after them, the exchange slots in
// which the second warp of a quadrant hands its row statistics to the first (32 x float2 each),
// and per quadrant the slot's full / empty mbarriers.
constexpr int kStageBytesPerWarp = 4096;
constexpr int kEpiStageBytes = kGemmEpiWarps * kStageBytesPerWarp;
constexpr int kEpiXchgSlots = 4 * 32 * 8;
constexpr int kEpiXchgBytes = kEpiXchgSlots + 4 * 2 * 8;
// Shared memory outside the operand ring: staging, exchange, 1 KB alignment slack, barriers.
constexpr int kGemmFixedSmem = kEpiStageBytes + kEpiXchgBytes + 1024 + 256;
constexpr int kMaxDynSmem = 227 * 1024;
__host__ __device__ constexpr int gemm_stages(int BN) {
  return ((kMaxDynSmem - kGemmFixedSmem) / gemm_stage_bytes(BN)) > 8
             ? 8
             : ((kMaxDynSmem - kGemmFixedSmem) / gemm_stage_bytes(BN));
}
__host__ __device__ constexpr int gemm_smem_bytes(int BN) {
  return gemm_stages(BN) * gemm_stage_bytes(BN) + kGemmFixedSmem;
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

// Chan's parallel merge of (count, mean, M2) statistics.
__device__ __forceinline__ void chan_merge(float& n_a, float& mean_a, float& m2_a, float n_b,
                                           float mean_b, float m2_b) {
  const float n = n_a + n_b;
  const float delta = mean_b - mean_a;
  const float f = n_b / n;
  mean_a = fmaf(delta, f, mean_a);
  m2_a = m2_a + m2_b + delta * delta * n_a * f;
  n_a = n;
}

// Epilogue of one 128 x BN accumulator held in TMEM (this warp's 32 lanes starting at t_row,
// output rows m_base .. m_base+31, the 32-column chunks c = 32 * (half + 2 j)): LayerNorm fold,
// alpha scaling, bias / per-image bias / SiLU / GEGLU / residual, optional row statistics of the
// stored values (the half-1 warp hands its statistics to the half-0 warp of the same quadrant
// through the slot `xchg` guarded by the mbarriers xbar[0] (full) / xbar[1] (empty); xphase counts
// the hand-offs).  Returns false when a bounded wait gave up.  Each 32-column chunk leaves
// through the warp's shared-memory staging buffer (swizzled so that row-per-thread writes and
// the bulk copy are bank-conflict free) as one TMA bulk store of 32 rows x 32 columns (16 for
// GEGLU); the residual chunk is read with coalesced 16-byte loads and transposed through the same
// buffer.  Rows >= M are clipped by the store.
// What epilogue_prefetch fetched for a tile.
struct EpiPre {
  bool res = false;       // fp16 residual of chunks 0 and 1 in staging buffers 0 and 1
  bool res3 = false;      // fp16 residual of the warp's third chunk in r3 (this lane's row)
  uint4 r3[4];
  bool uv = false;        // LayerNorm-fold vectors u, v of chunks 0 and 1 in buffers 0 and 1
  bool ln_ready = false;  // this row's LayerNorm mean / rstd below
  float ln_mean = 0.0f, ln_rstd = 1.0f;
};

// Issued by each epilogue warp before it waits for the tile's accumulator, so that the epilogue's
// inputs arrive while the tensor core still works on the tile: the row's LayerNorm statistics are
// merged, and the fp16 residual (coalesced 64-byte rows, in the swizzled staging layout) or the
// LayerNorm-fold vectors u, v (128 bytes each at the start of the buffer) of the warp's first two
// chunks are copied with cp.async into its two staging buffers, which the chunks' outputs reuse
// after reading them.  (Prefetching the bias lines into L1 measured slower.)
template <int BN, unsigned FL>
__device__ __forceinline__ EpiPre epilogue_prefetch(const GemmParams& p, int row, int n0, int m_base,
                                                    int half, uint8_t* stage, bool r3_ok = false) {
  const unsigned fl = epi_flags(FL, p.flags);
  EpiPre pre;
  const int lane = threadIdx.x & 31;
  const bool geglu = (fl & DLM_EPI_GEGLU) != 0;
  const bool lnf = (fl & kEpiLnFold) != 0;
  if (lnf) {
    if (row < p.M) {
      float cnt = 0.0f, mean = 0.0f, m2 = 0.0f;
      const float2* st = p.stats_in + static_cast<size_t>(row) * p.stats_in_parts;
      for (int i = 0; i < p.stats_in_parts; ++i) {
        const int c = min(p.stats_in_tile, p.ln_C - i * p.stats_in_tile);
        const float2 v = st[i];
        if (i == 0) {
          cnt = static_cast<float>(c);
          mean = v.x;
          m2 = v.y;
        } else {
          chan_merge(cnt, mean, m2, static_cast<float>(c), v.x, v.y);
        }
      }
      pre.ln_mean = mean;
      pre.ln_rstd = rsqrtf(fmaxf(m2 / static_cast<float>(p.ln_C), 0.0f) + p.ln_eps);
    }
    pre.ln_ready = true;
  }
  const bool resid16 = (fl & DLM_EPI_RESID) && !(fl & kEpiResidF32) && !geglu &&
                       !(fl & kEpiOutF32);
  if ((!resid16 && !lnf) || ((p.N - n0) & 31) != 0) return pre;
  // the bulk stores of the previous tile must have finished reading the staging buffers
  if (lane == 0) bulk_wait_read_le0();
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int n = n0 + 32 * half + 64 * j;
    if (32 * half + 64 * j >= BN || n >= p.N) break;
    uint8_t* buf = stage + j * 2048;
    if (resid16) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = (lane >> 2) + 8 * i, q = lane & 3;
        const int grow = m_base + rr;
        const __half* src = p.resid + static_cast<size_t>(grow < p.M ? grow : 0) * p.ldr + n + q * 8;
        cp_async16(buf + rr * 64 + ((q ^ ((rr >> 1) & 3)) * 16), src, grow < p.M ? 16u : 0u);
      }
    } else if (lane < 16) {
      const float* src = (lane < 8 ? p.ln_u : p.ln_v) + n + 4 * (lane & 7);
      cp_async16(buf + 16 * lane, src, 16u);
    }
  }
  // the third chunk's residual row straight into registers (64 contiguous bytes per lane: whole
  // 32-byte sectors; plain loads, since the residual may be the output itself).  Only the CTA-pair
  // kernel asks for it: its tiles are single-wave linears whose epilogue is exposed, and the
  // single-CTA kernel has no registers to spare.
  if (r3_ok && resid16 && 32 * half + 128 < BN && n0 + 32 * half + 128 < p.N) {
    const uint4* src = reinterpret_cast<const uint4*>(p.resid + static_cast<size_t>(row < p.M ? row : 0) * p.ldr +
                                                      n0 + 32 * half + 128);
#pragma unroll
    for (int q = 0; q < 4; ++q) pre.r3[q] = row < p.M ? src[q] : make_uint4(0, 0, 0, 0);
    pre.res3 = true;
  }
  cp_async_commit();
  pre.res = resid16;
  pre.uv = !resid16;
  return pre;
}

template <int BN, unsigned FL>
__device__ __forceinline__ bool epilogue_tile(const GemmParams& p, uint32_t t_row, int row, int n0,
                                              int m_base, uint8_t* stage, const CUtensorMap* tmC,
                                              int& sbuf, int half, float2* xchg, uint64_t* xbar,
                                              uint32_t& xphase, volatile int* abort_flag,
                                              const EpiPre& pre, int sk_c0 = 0, int sk_c1 = 0,
                                              int r_in_tile = 0) {
  const unsigned fl = epi_flags(FL, p.flags);
  const int lane = threadIdx.x & 31;
  // with inputs prefetched, chunk j (j < 2) of this tile uses staging buffer j
  const bool staged = pre.res || pre.uv;
  if (staged) sbuf = 0;
  int cj = 0;  // chunk index within this warp's chunks
  const bool row_ok = row < p.M;
  const bool geglu = (fl & DLM_EPI_GEGLU) != 0;
  float ln_mean = pre.ln_mean, ln_rstd = pre.ln_rstd;
  if ((fl & kEpiLnFold) && row_ok && !pre.ln_ready) {
    float cnt = 0.0f, mean = 0.0f, m2 = 0.0f;
    const float2* st = p.stats_in + static_cast<size_t>(row) * p.stats_in_parts;
    for (int i = 0; i < p.stats_in_parts; ++i) {
      const int c = min(p.stats_in_tile, p.ln_C - i * p.stats_in_tile);
      const float2 v = st[i];
      if (i == 0) {
        cnt = static_cast<float>(c);
        mean = v.x;
        m2 = v.y;
      } else {
        chan_merge(cnt, mean, m2, static_cast<float>(c), v.x, v.y);
      }
    }
    ln_mean = mean;
    ln_rstd = rsqrtf(fmaxf(m2 / static_cast<float>(p.ln_C), 0.0f) + p.ln_eps);
  }
  const int img = (row_ok ? row : p.M - 1) / p.rows_per_img;
  float s_cnt = 0.0f, s_mean = 0.0f, s_m2 = 0.0f;  // row statistics of this tile's outputs
#pragma unroll 1
  for (int c = 32 * half; c < BN; c += 64) {
    if (n0 + c >= p.N) break;
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    // stream-K owner: add the other CTAs' partial accumulators of this row, in CTA order
    for (int cc = sk_c0; cc < sk_c1; ++cc) {
      const float4* src = reinterpret_cast<const float4*>(
          p.sk_ws + (static_cast<size_t>(cc) * kGemmBM + r_in_tile) * BN + c);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t4 = __ldcg(src + j);
        v[4 * j] += t4.x;
        v[4 * j + 1] += t4.y;
        v[4 * j + 2] += t4.z;
        v[4 * j + 3] += t4.w;
      }
    }
    if (p.alpha != 1.0f) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
    }
    const int n = n0 + c;
    const bool pref = staged && cj < 2;
    if (pref && cj == 0) {
      cp_async_wait_all();
      __syncwarp();
    }
    if (fl & kEpiLnFold) {
      // v = rstd * (v - mean * u) + w, two columns per packed f32x2 FMA (same roundings)
      const float4* su = reinterpret_cast<const float4*>(stage + cj * 2048);
      const uint64_t nm2 = f2_pack(-ln_mean, -ln_mean), r2 = f2_pack(ln_rstd, ln_rstd);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 u4 = (pre.uv && cj < 2) ? su[j / 4] : __ldg(reinterpret_cast<const float4*>(p.ln_u + n + j));
        const float4 w4 = (pre.uv && cj < 2) ? su[8 + j / 4] : __ldg(reinterpret_cast<const float4*>(p.ln_v + n + j));
        uint64_t a0 = f2_fma(nm2, f2_pack(u4.x, u4.y), f2_pack(v[j], v[j + 1]));
        uint64_t a1 = f2_fma(nm2, f2_pack(u4.z, u4.w), f2_pack(v[j + 2], v[j + 3]));
        a0 = f2_fma(r2, a0, f2_pack(w4.x, w4.y));
        a1 = f2_fma(r2, a1, f2_pack(w4.z, w4.w));
        f2_unpack(a0, v[j], v[j + 1]);
        f2_unpack(a1, v[j + 2], v[j + 3]);
      }
    }
    if (fl & DLM_EPI_BIAS) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        float b[8];
        load_half8(p.bias + n + j, b);
#pragma unroll
        for (int q = 0; q < 8; q += 2) {
          const uint64_t t = f2_add(f2_pack(v[j + q], v[j + q + 1]), f2_pack(b[q], b[q + 1]));
          f2_unpack(t, v[j + q], v[j + q + 1]);
        }
      }
    }
    if (fl & DLM_EPI_BIAS2D) {
      const __half* b2 = p.bias2d + static_cast<size_t>(img) * p.ldb2 + n;
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        float b[8];
        load_half8(b2 + j, b);
#pragma unroll
        for (int q = 0; q < 8; q += 2) {
          const uint64_t t = f2_add(f2_pack(v[j + q], v[j + q + 1]), f2_pack(b[q], b[q + 1]));
          f2_unpack(t, v[j + q], v[j + q + 1]);
        }
      }
    }
    if (fl & DLM_EPI_SILU) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
    }
    uint8_t* buf = stage + sbuf * 2048;
    if (!pref) {
      // the bulk store that last used this buffer must have finished reading it
      if (lane == 0) bulk_wait_read_le1();
    }
    __syncwarp();
    if (geglu) {
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float g0, g1;
        gelu_erf_x2(v[4 * j + 1], v[4 * j + 3], g0, g1);
        const float a0 = v[4 * j] * g0;
        const float a1 = v[4 * j + 2] * g1;
        o[j] = pack_half2(a0, a1);
      }
      // 32-byte rows, 32-byte swizzle: 16-byte chunk q of row r at q ^ ((r >> 2) & 1)
      uint8_t* rb = buf + lane * 32;
      const int sw = (lane >> 2) & 1;
      *reinterpret_cast<uint4*>(rb + ((0 ^ sw) * 16)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(rb + ((1 ^ sw) * 16)) = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
      // 64-byte rows, 64-byte swizzle: 16-byte chunk q of row r at q ^ ((r >> 1) & 3)
      if ((fl & DLM_EPI_RESID) && (fl & kEpiResidF32)) {
        if (row_ok) {
          const float* rs = reinterpret_cast<const float*>(p.resid) + static_cast<size_t>(row) * p.ldr + n;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 t = *reinterpret_cast<const float4*>(rs + j);
            v[j] += p.resid_scale * t.x;
            v[j + 1] += p.resid_scale * t.y;
            v[j + 2] += p.resid_scale * t.z;
            v[j + 3] += p.resid_scale * t.w;
          }
        }
      } else if (fl & DLM_EPI_RESID) {
        if (pre.res3 && cj == 2) {
          const uint64_t rs2 = f2_pack(p.resid_scale, p.resid_scale);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __half2* h = reinterpret_cast<const __half2*>(&pre.r3[q]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 t = __half22float2(h[k]);
              const uint64_t r = f2_fma(rs2, f2_pack(t.x, t.y), f2_pack(v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]));
              f2_unpack(r, v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]);
            }
          }
        } else {
        if (!(pre.res && cj < 2)) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = (lane >> 2) + 8 * i, q = lane & 3;
            const int grow = m_base + rr;
            uint4 u = make_uint4(0, 0, 0, 0);
            if (grow < p.M)
              u = *reinterpret_cast<const uint4*>(p.resid + static_cast<size_t>(grow) * p.ldr + n + q * 8);
            *reinterpret_cast<uint4*>(buf + rr * 64 + ((q ^ ((rr >> 1) & 3)) * 16)) = u;
          }
          __syncwarp();
        }
        const uint64_t rs2 = f2_pack(p.resid_scale, p.resid_scale);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = *reinterpret_cast<const uint4*>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) * 16));
          const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 t = __half22float2(h[k]);
            const uint64_t r = f2_fma(rs2, f2_pack(t.x, t.y), f2_pack(v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]));
            f2_unpack(r, v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]);
          }
        }
        __syncwarp();
        }
      }
      if (fl & kEpiOutF32) {
        // fp32 output: two halves of 16 columns, each 32 rows x 64 bytes through one staging
        // buffer and one bulk store (the second half uses the other buffer)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint8_t* hb = stage + sbuf * 2048;
          if (h == 1) {
            if (lane == 0) bulk_wait_read_le1();
            __syncwarp();
          }
          uint8_t* rb = hb + lane * 64;
          const int sw = (lane >> 1) & 3;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4*>(rb + ((q ^ sw) * 16)) =
                make_float4(v[16 * h + 4 * q], v[16 * h + 4 * q + 1], v[16 * h + 4 * q + 2],
                            v[16 * h + 4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(tmC, hb, n + 16 * h, m_base);
            bulk_commit_group();
          }
          sbuf ^= 1;
        }
        continue;
      }
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] = pack_half2(v[2 * j], v[2 * j + 1]);
      uint8_t* rb = buf + lane * 64;
      const int sw = (lane >> 1) & 3;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(rb + ((q ^ sw) * 16)) =
            make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      if ((fl & kEpiRowStats) && row_ok) {
        // statistics of the values as stored (fp16), chunk by chunk, merged with Chan's formula
        float f[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&o[j]));
          f[2 * j] = t.x;
          f[2 * j + 1] = t.y;
        }
        // two interleaved partial sums per packed f32x2 add / FMA
        uint64_t s2 = f2_pack(f[0], f[1]);
#pragma unroll
        for (int j = 2; j < 32; j += 2) s2 = f2_add(s2, f2_pack(f[j], f[j + 1]));
        float s_lo, s_hi;
        f2_unpack(s2, s_lo, s_hi);
        const float cm = (s_lo + s_hi) * (1.0f / 32.0f);
        const uint64_t ncm = f2_pack(-cm, -cm);
        uint64_t q2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const uint64_t d = f2_add(f2_pack(f[j], f[j + 1]), ncm);
          q2 = f2_fma(d, d, q2);
        }
        float q_lo, q_hi;
        f2_unpack(q2, q_lo, q_hi);
        const float m2 = q_lo + q_hi;
        if (s_cnt == 0.0f) {
          s_cnt = 32.0f;
          s_mean = cm;
          s_m2 = m2;
        } else {
          chan_merge(s_cnt, s_mean, s_m2, 32.0f, cm, m2);
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, buf, geglu ? (n >> 1) : n, m_base);
      bulk_commit_group();
    }
    sbuf ^= 1;
    ++cj;
  }
  if (fl & kEpiRowStats) {
    const uint32_t ph = xphase & 1;
    ++xphase;
    if (half == 1) {
      if (!mbar_wait(&xbar[1], ph ^ 1, abort_flag, p.status, kDevTimeoutEpilogue)) return false;
      xchg[lane] = make_float2(s_mean, s_m2);
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[0]);
    } else {
      if (!mbar_wait(&xbar[0], ph, abort_flag, p.status, kDevTimeoutEpilogue)) return false;
      const float2 o = xchg[lane];
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[1]);
      // the half-1 warp stored the chunks c = 32, 96, ... below BN and N - n0 (32 values each)
      float cnt1 = 0.0f;
      for (int c = 32; c < BN && n0 + c < p.N; c += 64) cnt1 += 32.0f;
      if (cnt1 > 0.0f) {
        if (s_cnt == 0.0f) {
          s_cnt = cnt1;
          s_mean = o.x;
          s_m2 = o.y;
        } else {
          chan_merge(s_cnt, s_mean, s_m2, cnt1, o.x, o.y);
        }
      }
      if (row_ok) p.stats_out[static_cast<size_t>(row) * p.stats_ld + n0 / BN] = make_float2(s_mean, s_m2);
    }
  }
  return true;
}

// Stream-K contributor: this CTA's fp32 partial accumulator of its 32 rows of a cut tile, to its
// workspace slot sk_ws[blockIdx.x] (128 contiguous bytes per lane and 32-column chunk).
template <int BN>
__device__ __forceinline__ void epilogue_partial(const GemmParams& p, uint32_t t_row, int r_in_tile,
                                                 int half) {
  float* dst = p.sk_ws + (static_cast<size_t>(blockIdx.x) * kGemmBM + r_in_tile) * BN;
#pragma unroll 1
  for (int c = 32 * half; c < BN; c += 64) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_row + c, r);
    tmem_ld_wait();
    float4* d4 = reinterpret_cast<float4*>(dst + c);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      __stcg(d4 + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
  }
}

template <int BN, unsigned FL>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
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
  uint8_t* sEpi = sB + STAGES * B_BYTES;  // 1024-aligned: stage sizes are multiples of 1 KB
  float2* sXchg = reinterpret_cast<float2*>(sEpi + kEpiStageBytes);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(sEpi + kEpiStageBytes + kEpiXchgSlots);
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kEpiStageBytes + kEpiXchgBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* sk_bar = tempty + 2;  // stream-K: the four epilogue warps meet here
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sk_bar + 1);
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
      mbar_init(&tempty[a], kGemmEpiWarps);
    }
    mbar_init(sk_bar, kGemmEpiWarps);
    for (int x = 0; x < 8; ++x) mbar_init(&xbar[x], 1);
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
  griddep_wait();  // inputs of this GEMM are written by the previous kernel

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      SegIter si;
      si.init(p);
      TileSeg sg;
      while (ok && si.next(p, sg)) {
        const int m0 = (sg.tile / p.n_tiles) * kGemmBM;
        const int n0 = (sg.tile % p.n_tiles) * BN;
        if (p.amode == 0) {
          for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
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
          // k-block kb0 -> (segment, tap, channel block); K order is (segment, tap, channel)
          int sidx = 0, base = 0;
          while (sidx < p.nseg - 1 &&
                 base + (p.seg[sidx].kind == 1 ? 1 : 9) * p.seg[sidx].cblocks <= sg.kb0) {
            base += (p.seg[sidx].kind == 1 ? 1 : 9) * p.seg[sidx].cblocks;
            ++sidx;
          }
          int tap = (sg.kb0 - base) / p.seg[sidx].cblocks;
          int cb = (sg.kb0 - base) - tap * p.seg[sidx].cblocks;
          for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
            const ConvSeg cs = p.seg[sidx];
            const CUtensorMap* am = cs.map == 0 ? &tmA0 : (cs.map == 1 ? &tmA1 : &tmA2);
            const int kh = tap / 3, kw = tap - (tap / 3) * 3;
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
            uint8_t* dstA = sA + stage * A_BYTES;
            if (cs.kind == 0) {
              tma_load_4d(dstA, am, &full[stage], cb * 64, ow0 + kw - 1, oh0 + kh - 1, img);
            } else if (cs.kind == 1) {
              tma_load_4d(dstA, am, &full[stage], cb * 64, ow0, oh0, img);
            } else {
              // input row 2*oh + kh - 1: kh=0 -> odd plane, row oh-1; kh=1 -> even, oh;
              // kh=2 -> odd, oh.  Same for columns.
              const int pr = (kh == 1) ? 0 : 1, dr = (kh == 0) ? -1 : 0;
              const int pc = (kw == 1) ? 0 : 1, dc = (kw == 0) ? -1 : 0;
              tma_load_5d(dstA, am, &full[stage], cb * 64, ow0 + dc, oh0 + dr, img, pr * 2 + pc);
            }
            tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * kGemmBK, n0);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            if (++cb == cs.cblocks) {
              cb = 0;
              if (++tap == (cs.kind == 1 ? 1 : 9)) {
                tap = 0;
                ++sidx;
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
      SegIter si;
      si.init(p);
      TileSeg sg;
      while (ok && si.next(p, sg)) {
        const int acc = i & 1;
        const uint32_t acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tbase + static_cast<uint32_t>(acc * BN);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
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
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb != sg.kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
        ++i;
      }
      // the last MMA is issued: the next kernel may launch during this CTA's final epilogue
      griddep_launch_dependents();
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r_in_tile = quad * 32 + lane;
    int sbuf = 0;
    int i = 0;
    uint32_t sk_phase = 0, xphase = 0;
    SegIter si;
    si.init(p);
    TileSeg sg;
    // the epilogue warps meet (bounded) before a stream-K flag changes hands
    auto sk_meet = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(sk_bar);
      const bool okm = mbar_wait(sk_bar, sk_phase, abort_flag, p.status, kDevTimeoutEpilogue);
      sk_phase ^= 1;
      return okm;
    };
    bool ok = true;
    while (ok && si.next(p, sg)) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      const int m0 = (sg.tile / p.n_tiles) * kGemmBM;
      const int n0 = (sg.tile % p.n_tiles) * BN;
      const int row = m0 + r_in_tile;
      uint8_t* stage_buf = sEpi + (warp - 2) * kStageBytesPerWarp;
      const EpiPre pre = (p.sk_ctas > 0 && sg.kb0 > 0)
                             ? EpiPre{}
                             : epilogue_prefetch<BN, FL>(p, row, n0, m0 + quad * 32, half, stage_buf);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tbase + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      if (p.sk_ctas > 0 && sg.kb0 > 0) {
        // contributor: hand the partial accumulator to the tile's owner
        epilogue_partial<BN>(p, t_row, r_in_tile, half);
        __threadfence();
        ok = sk_meet();
        if (ok && warp == 2 && lane == 0) {
          __threadfence();
          flag_store_release(p.sk_flags + blockIdx.x, 1);
        }
      } else {
        int c0 = blockIdx.x + 1, c1 = c0;
        if (p.sk_ctas > 0 && sg.kb1 < p.num_kb) {
          // owner of a cut tile: its contributors are the following CTAs whose ranges start
          // inside it
          const long long tile_end = static_cast<long long>(sg.tile + 1) * p.num_kb;
          while (c1 < p.sk_ctas) {
            long long a, b;
            sk_range(p, c1, a, b);
            if (a >= tile_end) break;
            ++c1;
          }
          for (int cc = c0; cc < c1 && ok; ++cc)
            ok = flag_wait_acquire(p.sk_flags + cc, 1, abort_flag, p.status, kDevTimeoutStreamK);
        }
        if (ok) {
          ok = epilogue_tile<BN, FL>(p, t_row, row, n0, m0 + quad * 32, stage_buf, &tmC, sbuf, half,
                                 sXchg + quad * 32, xbar + 2 * quad, xphase, abort_flag, pre,
                                 c0, c1, r_in_tile);
          if (ok && c1 > c0) {
            // every warp has read the partials: clear the flags for the next launch
            ok = sk_meet();
            if (ok && warp == 2)
              for (int cc = c0 + lane; cc < c1; cc += 32) p.sk_flags[cc] = 0;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      ++i;
    }
    // the staging buffers must have been read before the CTA exits; the stores themselves
    // complete with the grid (a dependent grid's griddepcontrol.wait covers them)
    if (lane == 0) bulk_wait_read_le0();
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


// ======================================================================================
// CTA-pair variant (tcgen05 cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x BN tile.  Each CTA TMA-loads its own 128 rows of A and its half (BN/2 rows) of B into
// its own shared memory; the bulk copies of both CTAs complete on the even CTA's `full` barrier;
// the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = BN) and commits to the `empty` and
// `tfull` barriers of both CTAs (multicast commit).  Each CTA's TMEM holds its 128 rows of the
// accumulator (two buffers of BN columns); each CTA runs the epilogue for its rows and both signal
// the even CTA's `tempty`.  Per SM this moves half of B through L2 and shared memory compared with
// the single-CTA kernel, which is what lets the tensor core run at full rate for BN = 256.
// A ring stage holds two 64-wide k-blocks (kPairKsub), so the issuing thread waits, commits and
// advances once per 8 MMAs: its per-stage bookkeeping (~450 clocks on B200, whatever N is) then
// costs less than the tensor work of the stage for BN >= 160.  An odd k-block count leaves the
// last stage of a tile half full.
// Loads carry no multicast qualifier: every CTA fetches its own operands.
// ======================================================================================

constexpr int kPairKsub = 2;
__host__ __device__ constexpr int gemm2_stage_bytes(int BN) {
  return kPairKsub * (kGemmBM + BN / 2) * kGemmBK * 2;
}
__host__ __device__ constexpr int gemm2_stages(int BN) {
  return ((kMaxDynSmem - kGemmFixedSmem) / gemm2_stage_bytes(BN)) > 8
             ? 8
             : ((kMaxDynSmem - kGemmFixedSmem) / gemm2_stage_bytes(BN));
}
__host__ __device__ constexpr int gemm2_smem_bytes(int BN) {
  return gemm2_stages(BN) * gemm2_stage_bytes(BN) + kGemmFixedSmem;
}

template <int BN, unsigned FL>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                    const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  constexpr int BNH = BN / 2;
  constexpr int A_SUB = kGemmBM * kGemmBK * 2;  // one 64-wide k-block of A (this CTA's rows)
  constexpr int B_SUB = BNH * kGemmBK * 2;      // one k-block of this CTA's half of B
  constexpr int A_BYTES = kPairKsub * A_SUB;    // per ring stage
  constexpr int B_BYTES = kPairKsub * B_SUB;
  constexpr int STAGES = gemm2_stages(BN);
  constexpr uint32_t TMEM_COLS = gemm_tmem_cols(BN);
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair UMMA N");
  static_assert(BNH % 8 == 0, "B half must hold whole 8-row swizzle atoms");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sEpi = sB + STAGES * B_BYTES;  // 1024-aligned: stage sizes are multiples of 1 KB
  float2* sXchg = reinterpret_cast<float2*>(sEpi + kEpiStageBytes);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(sEpi + kEpiStageBytes + kEpiXchgSlots);
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kEpiStageBytes + kEpiXchgBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kGemmEpiWarps);  // the epilogue warps of both CTAs
    }
    for (int x = 0; x < 8; ++x) mbar_init(&xbar[x], 1);
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
    tmem_alloc2(tmem_slot, TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  griddep_wait();  // inputs of this GEMM are written by the previous kernel
  const int num_tiles = p.m_tiles * p.n_tiles;  // m tiles of 256 rows

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        const int m0 = (t / p.n_tiles) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM;
        const int nb = (t % p.n_tiles) * BN + static_cast<int>(rank) * BNH;
        if (p.amode == 0) {
          // dense A: one wait / expect_tx per ring stage, then its k-blocks' A and B boxes (the
          // thread's per-k-block work bounds short tiles, so this path stays minimal)
          for (int kb = 0; kb < p.num_kb; kb += kPairKsub) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
              ok = false;
              break;
            }
            const int nsub = p.num_kb - kb >= kPairKsub ? kPairKsub : p.num_kb - kb;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * nsub * (A_SUB + B_SUB));
            const uint32_t fb = pair_leader_addr(&full[stage]);
            for (int su = 0; su < nsub; ++su) {
              tma2_load_2d(sA + stage * A_BYTES + su * A_SUB, &tmA0, fb, (kb + su) * kGemmBK, m0);
              tma2_load_2d(sB + stage * B_BYTES + su * B_SUB, &tmB, fb, (kb + su) * kGemmBK, nb);
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          continue;
        }
        int img = 0, oh0 = 0, ow0 = 0;
        if (p.amode == 1) {
          const int hw = p.oH * p.oW;
          img = m0 / hw;
          const int rem = m0 - img * hw;
          oh0 = rem / p.oW;
          ow0 = rem - oh0 * p.oW;
        }
        int kb = 0;
        int sub = 0;  // k-block within the ring stage
        const int nseg = p.amode == 0 ? 1 : p.nseg;
        for (int s = 0; s < nseg && ok; ++s) {
          const ConvSeg sg = p.seg[s];
          const CUtensorMap* am = p.amode == 0 ? &tmA0 : (sg.map == 0 ? &tmA0 : (sg.map == 1 ? &tmA1 : &tmA2));
          const int ntaps = p.amode == 0 ? 1 : (sg.kind == 1 ? 1 : 9);
          const int ncb = p.amode == 0 ? p.num_kb : sg.cblocks;
          for (int tap = 0; tap < ntaps && ok; ++tap) {
            const int kh = tap / 3, kw = tap - (tap / 3) * 3;
            for (int cb = 0; cb < ncb; ++cb) {
              if (sub == 0) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
                  ok = false;
                  break;
                }
                const int nsub = p.num_kb - kb >= kPairKsub ? kPairKsub : p.num_kb - kb;
                if (leader) mbar_arrive_expect_tx(&full[stage], 2 * nsub * (A_SUB + B_SUB));
              }
              const uint32_t fb = pair_leader_addr(&full[stage]);
              uint8_t* dstA = sA + stage * A_BYTES + sub * A_SUB;
              if (p.amode == 0) {
                tma2_load_2d(dstA, am, fb, cb * kGemmBK, m0);
              } else if (sg.kind == 0) {
                tma2_load_4d(dstA, am, fb, cb * 64, ow0 + kw - 1, oh0 + kh - 1, img);
              } else if (sg.kind == 1) {
                tma2_load_4d(dstA, am, fb, cb * 64, ow0, oh0, img);
              } else {
                const int pr = (kh == 1) ? 0 : 1, dr = (kh == 0) ? -1 : 0;
                const int pc = (kw == 1) ? 0 : 1, dc = (kw == 0) ? -1 : 0;
                tma2_load_5d(dstA, am, fb, cb * 64, ow0 + dc, oh0 + dr, img, pr * 2 + pc);
              }
              tma2_load_2d(sB + stage * B_BYTES + sub * B_SUB, &tmB, fb, kb * kGemmBK, nb);
              ++kb;
              if (++sub == kPairKsub || kb == p.num_kb) {
                sub = 0;
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
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * kGemmBM, BN, false);
      // Descriptors of stage 0 as low words over one high word; the ring is walked one pass at a
      // time with the stage index unrolled, so barrier addresses and descriptor offsets are
      // immediates: this thread's bookkeeping per stage is what bounds short MMAs.
      const uint64_t da0 = sw128_desc(smem_u32(sA), 16, 1024);
      const uint32_t a_lo0 = static_cast<uint32_t>(da0);
      const uint32_t b_lo0 = static_cast<uint32_t>(sw128_desc(smem_u32(sB), 16, 1024));
      const uint32_t d_hi = static_cast<uint32_t>(da0 >> 32);
      uint32_t phase = 0;
      int i = 0;
      int t = pair;
      int kb = 0;
      bool ok = true;
      bool have = t < num_tiles;
      uint32_t d_tmem = tbase;
      while (have && ok) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) {
          if (have && ok) {
            if (kb == 0) {
              const int acc = i & 1;
              if (mbar_wait(&tempty[acc], ((i >> 1) & 1) ^ 1, abort_flag, p.status, kDevTimeoutMma)) {
                tc_fence_after();
                d_tmem = tbase + static_cast<uint32_t>(acc * BN);
              } else {
                ok = false;
              }
            }
            if (ok && !mbar_wait(&full[st], phase, abort_flag, p.status, kDevTimeoutMma)) ok = false;
            if (ok) {
              tc_fence_after();
#pragma unroll
              for (int sub = 0; sub < kPairKsub; ++sub) {
                const uint32_t a_off = static_cast<uint32_t>(st * A_BYTES + sub * A_SUB) >> 4;
                const uint32_t b_off = static_cast<uint32_t>(st * B_BYTES + sub * B_SUB) >> 4;
                if (sub == 0 || kb + sub < p.num_kb) {
                  umma2_f16_ss_lo(d_tmem, a_lo0 + a_off, b_lo0 + b_off, d_hi, idesc,
                                  (kb + sub) != 0 ? 1u : 0u);
#pragma unroll
                  for (int k = 1; k < kGemmBK / 16; ++k)
                    umma2_f16_ss_lo(d_tmem, a_lo0 + a_off + 2 * k, b_lo0 + b_off + 2 * k, d_hi, idesc, 1u);
                }
              }
              umma2_commit_mc(&empty[st], 0x3);
              kb += kPairKsub;
              if (kb >= p.num_kb) {
                umma2_commit_mc(&tfull[i & 1], 0x3);
                ++i;
                kb = 0;
                t += npairs;
                have = t < num_tiles;
              }
            }
          }
        }
        phase ^= 1;
      }
      griddep_launch_dependents();
    } else if (lane == 0) {
      griddep_launch_dependents();  // the pair's trigger is the even CTA's
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    int sbuf = 0;
    int i = 0;
    uint32_t xphase = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++i) {
      const int acc = i & 1;
      const uint32_t acc_phase = (i >> 1) & 1;
      const int m0 = (t / p.n_tiles) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM;
      const int n0 = (t % p.n_tiles) * BN;
      const int row = m0 + quad * 32 + lane;
      uint8_t* stage_buf = sEpi + (warp - 2) * kStageBytesPerWarp;
      const EpiPre pre = epilogue_prefetch<BN, FL>(p, row, n0, m0 + quad * 32, half, stage_buf, true);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tbase + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      if (!epilogue_tile<BN, FL>(p, t_row, row, n0, m0 + quad * 32, stage_buf, &tmC, sbuf, half,
                             sXchg + quad * 32, xbar + 2 * quad, xphase, abort_flag, pre))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&tempty[acc], 0);
    }
    // the staging buffers must have been read before the CTA exits; the stores themselves
    // complete with the grid (a dependent grid's griddepcontrol.wait covers them)
    if (lane == 0) bulk_wait_read_le0();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tbase, TMEM_COLS);
  }
}

}  // namespace dlm
