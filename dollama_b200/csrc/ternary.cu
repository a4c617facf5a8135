// BitNet ternary-weight x int8-activation linear (the tag LM's BitLinear), bit-exact with the
// reference's integer path (src/models/bitnet.hpp: quantize_weight_ternary :70-109,
// quantize_activation_int8 :123-165, BitNet::bitlinear :447-471).
//
// Weights are quantized once (per output row: alpha = mean|w| in double, q = clamp(round(w/alpha),
// -1, 1)) and stored as 2-bit codes, 16 per 32-bit word (00 = 0, 01 = +1, 11 = -1), i.e. 1/16 of
// the fp32 bytes; activations are quantized per token (scale = max|x|/127, q = clamp(round(x/scale),
// -127, 127)).  Both quantizers run in double with explicit round-to-nearest operations, in the
// same order as the reference, so codes and scales are identical.
//
// The GEMM keeps the reference's exact arithmetic: int32 accumulation (|acc| <= 127 * K fits for
// K < 2^24) and y = float(double(acc) * double(alpha_n) * double(scale_m)), on three paths that
// give the same bits: the tensor cores (tcgen05.mma kind::i8) in 128 x 128 tiles for prefill-sized
// inputs (ternary_gemm_tc_kernel), in 128 x 32 / 64 tiles for decode-sized ones
// (ternary_gemm_tcd_kernel), and dp4a for the remaining shapes (ternary_gemm_kernel: a 32-token x
// 64-output tile per CTA, 32 outputs when 64-wide tiles would leave most SMs idle; K runs in
// chunks of 256 whose packed weights and activations arrive by asynchronous copies while the
// previous chunk is multiplied; the weight chunk is expanded to int8 once in shared memory, rows
// padded by 16 bytes so 16-byte reads of consecutive rows hit distinct banks, and amortised over
// the 32 tokens; the inner loop is 16-byte shared loads + dp4a).
#include <cstdint>
#include <cstdlib>

#include "ptx.cuh"
#include "ternary.h"

namespace dlm {

namespace {

constexpr int kTM = 32;       // tokens per CTA
constexpr int kTN = 64;       // outputs per CTA (or 32, see ternary_gemm_i8)
constexpr int kKC = 256;      // K chunk (elements)
constexpr int kRow = kKC + 16;  // padded smem row (bytes)
constexpr int kThreads = 256;
// Token rows from which the tensor-core path is used (DLM_TERNARY_TC_ROWS overrides, for
// measurements).
// The decode tensor-core path (DLM_TERNARY_TCD=0 keeps dp4a for every decode-sized call).
bool tcd_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("DLM_TERNARY_TCD");
    return !(e && e[0] == '0');
  }();
  return v;
}

int tc_min_rows() {
  static const int v = [] {
    const char* e = std::getenv("DLM_TERNARY_TC_ROWS");
    return e ? std::atoi(e) : 1024;
  }();
  return v;
}

// One thread per output row: exact per-row ternary quantization, then 2-bit packing.
__global__ void ternary_pack_kernel(const float* __restrict__ w, int N, int K,
                                    uint32_t* __restrict__ packed, float* __restrict__ alpha) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float* row = w + static_cast<size_t>(n) * K;
  double sum_abs = 0.0;
  for (int i = 0; i < K; ++i) sum_abs = __dadd_rn(sum_abs, fabs(static_cast<double>(row[i])));
  const double a = __ddiv_rn(sum_abs, static_cast<double>(K));
  alpha[n] = static_cast<float>(a);
  const double inv = a == 0.0 ? 0.0 : __ddiv_rn(1.0, a);
  uint32_t* out = packed + static_cast<size_t>(n) * (K / 16);
  for (int w16 = 0; w16 < K / 16; ++w16) {
    uint32_t word = 0;
    for (int j = 0; j < 16; ++j) {
      uint32_t code = 0;
      if (a != 0.0) {
        double r = round(__dmul_rn(static_cast<double>(row[w16 * 16 + j]), inv));
        if (r > 1.0) r = 1.0;
        if (r < -1.0) r = -1.0;
        code = r > 0.0 ? 1u : (r < 0.0 ? 3u : 0u);
      }
      word |= code << (2 * j);
    }
    out[w16] = word;
  }
}

// Per-tensor alpha: sum |w| over the whole tensor in row-major order, one thread (load time only),
// so the double sum rounds exactly as a sequential loop.
__global__ void tensor_absmean_kernel(const float* __restrict__ w, size_t n, double* __restrict__ out) {
  double sum_abs = 0.0;
  for (size_t i = 0; i < n; ++i) sum_abs = __dadd_rn(sum_abs, fabs(static_cast<double>(w[i])));
  *out = __ddiv_rn(sum_abs, static_cast<double>(n));
}

// Packs every row with the given alpha (one thread per row).
__global__ void ternary_pack_alpha_kernel(const float* __restrict__ w, int N, int K,
                                          const double* __restrict__ alpha_in,
                                          uint32_t* __restrict__ packed, float* __restrict__ alpha) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const double a = *alpha_in;
  alpha[n] = static_cast<float>(a);
  const double inv = a == 0.0 ? 0.0 : __ddiv_rn(1.0, a);
  const float* row = w + static_cast<size_t>(n) * K;
  uint32_t* out = packed + static_cast<size_t>(n) * (K / 16);
  for (int w16 = 0; w16 < K / 16; ++w16) {
    uint32_t word = 0;
    for (int j = 0; j < 16; ++j) {
      uint32_t code = 0;
      if (a != 0.0) {
        double r = round(__dmul_rn(static_cast<double>(row[w16 * 16 + j]), inv));
        if (r > 1.0) r = 1.0;
        if (r < -1.0) r = -1.0;
        code = r > 0.0 ? 1u : (r < 0.0 ? 3u : 0u);
      }
      word |= code << (2 * j);
    }
    out[w16] = word;
  }
}

// One warp per token: exact absmax int8 quantization.
__global__ void quant_act_kernel(const float* __restrict__ x, int M, int K, int8_t* __restrict__ xq,
                                 float* __restrict__ xscale) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (m >= M) return;
  const float* row = x + static_cast<size_t>(m) * K;
  double amax = 0.0;
  for (int i = lane; i < K; i += 32) amax = fmax(amax, fabs(static_cast<double>(row[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmax(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const double scale = __ddiv_rn(amax, 127.0);
  const double inv = scale == 0.0 ? 0.0 : __ddiv_rn(1.0, scale);
  if (lane == 0) xscale[m] = static_cast<float>(scale);
  int8_t* q = xq + static_cast<size_t>(m) * K;
  for (int i = lane; i < K; i += 32) {
    int v = 0;
    if (scale != 0.0) {
      double r = round(__dmul_rn(static_cast<double>(row[i]), inv));
      if (r > 127.0) r = 127.0;
      if (r < -127.0) r = -127.0;
      v = static_cast<int>(r);
    }
    q[i] = static_cast<int8_t>(v);
  }
}

// 4 two-bit codes (one byte) -> 4 int8 lanes {0, +1, -1}.
__device__ __forceinline__ uint32_t decode4(uint32_t b) {
  const uint32_t t = (b & 0x03u) | ((b & 0x0Cu) << 6) | ((b & 0x30u) << 12) | ((b & 0xC0u) << 18);
  const uint32_t lo = t & 0x01010101u;
  const uint32_t hi = (t >> 1) & 0x01010101u;
  return lo | (hi * 0xFEu);
}

template <int TN, bool kRope>
__global__ void __launch_bounds__(kThreads)
    ternary_gemm_kernel(const uint32_t* __restrict__ wp, const float* __restrict__ alpha,
                        const int8_t* __restrict__ xq, const float* __restrict__ xscale,
                        float* __restrict__ y, int M, int N, int K, int accumulate, RopeQkv rp) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  constexpr int NI = TN / 16;  // outputs per thread
  __shared__ __align__(16) int8_t sw[TN * kRow];              // expanded int8 weight chunk
  __shared__ __align__(16) int8_t sx[2][kTM * kRow];          // activation chunks (double buffer)
  __shared__ __align__(16) uint32_t sp[2][TN * (kKC / 16)];   // packed weight chunks (double buffer)
  const int n0 = blockIdx.x * TN, m0 = blockIdx.y * kTM;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // outputs n0 + tx + 16i, tokens m0 + ty + 16j
  int acc[2][NI];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int i = 0; i < NI; ++i) acc[j][i] = 0;
  const int wwords = K / 16;
  // chunk [k0, k0 + kc) of the packed weights and activations into buffer `buf` by 16-byte
  // asynchronous copies (rows beyond N / M arrive as zeros); K % 64 == 0 keeps every source
  // 16-byte aligned
  auto fetch = [&](int k0, int buf) {
    const int kc = min(kKC, K - k0);
    const int wq = kc / 64;  // 16-byte pieces per packed row
    for (int idx = tid; idx < TN * wq; idx += kThreads) {
      const int r = idx / wq, c = idx - r * wq;
      const bool in = n0 + r < N;
      const uint32_t* src = in ? wp + static_cast<size_t>(n0 + r) * wwords + k0 / 16 + 4 * c : wp;
      cp_async16(&sp[buf][r * (kKC / 16) + 4 * c], src, in ? 16u : 0u);
    }
    const int xv = kc / 16;
    for (int idx = tid; idx < kTM * xv; idx += kThreads) {
      const int r = idx / xv, c = idx - r * xv;
      const bool in = m0 + r < M;
      const int8_t* src = in ? xq + static_cast<size_t>(m0 + r) * K + k0 + 16 * c : xq;
      cp_async16(sx[buf] + r * kRow + 16 * c, src, in ? 16u : 0u);
    }
    cp_async_commit();
  };
  fetch(0, 0);
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += kKC, buf ^= 1) {
    const int kc = min(kKC, K - k0);  // multiple of 64
    cp_async_wait_all();
    __syncthreads();  // chunk k0 landed for every thread; the previous chunk's reads are done
    // expand the packed chunk: TN rows x kc/16 words, four words (64 codes) per 16-byte piece
    const int wq = kc / 64;
    for (int idx = tid; idx < TN * wq; idx += kThreads) {
      const int r = idx / wq, c = idx - r * wq;
      const uint4 v = *reinterpret_cast<const uint4*>(&sp[buf][r * (kKC / 16) + 4 * c]);
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
      uint32_t* dst = reinterpret_cast<uint32_t*>(sw + r * kRow + c * 64);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t wd = words[q];
        dst[4 * q + 0] = decode4(wd & 0xFFu);
        dst[4 * q + 1] = decode4((wd >> 8) & 0xFFu);
        dst[4 * q + 2] = decode4((wd >> 16) & 0xFFu);
        dst[4 * q + 3] = decode4(wd >> 24);
      }
    }
    __syncthreads();  // expanded weights ready; packed buffer `buf` free
    if (k0 + kKC < K) fetch(k0 + kKC, buf ^ 1);  // lands while this chunk is multiplied
    const int8_t* sxb = sx[buf];
    for (int k = 0; k < kc; k += 16) {
      uint4 xv4[2], wv4[NI];
#pragma unroll
      for (int j = 0; j < 2; ++j) xv4[j] = *reinterpret_cast<const uint4*>(sxb + (ty + 16 * j) * kRow + k);
#pragma unroll
      for (int i = 0; i < NI; ++i) wv4[i] = *reinterpret_cast<const uint4*>(sw + (tx + 16 * i) * kRow + k);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          int a = acc[j][i];
          a = __dp4a(static_cast<int>(xv4[j].x), static_cast<int>(wv4[i].x), a);
          a = __dp4a(static_cast<int>(xv4[j].y), static_cast<int>(wv4[i].y), a);
          a = __dp4a(static_cast<int>(xv4[j].z), static_cast<int>(wv4[i].z), a);
          a = __dp4a(static_cast<int>(xv4[j].w), static_cast<int>(wv4[i].w), a);
          acc[j][i] = a;
        }
    }
  }
  if constexpr (kRope) {
    // q|k|v of one position per sequence: a 64-output tile is one head of q, k or v; this thread's
    // outputs tx, tx + 16, tx + 32, tx + 48 of it are the RoPE pairs (tx, tx + 32) and
    // (tx + 16, tx + 48) (bitnet.hpp:472-488), rotated in double from the float outputs
    static_assert(TN == 64, "one head per tile");
    const int base = *rp.pos;
    const int part = n0 / rp.D, hd = (n0 % rp.D) / kTN, H = rp.D / kTN;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int m = m0 + ty + 16 * j;
      if (m >= M) continue;
      const double sc = static_cast<double>(xscale[m]);
      float v[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i)
        v[i] = __double2float_rn(__dmul_rn(
            __dmul_rn(static_cast<double>(acc[j][i]), static_cast<double>(alpha[n0 + tx + 16 * i])), sc));
      const size_t cache = ((static_cast<size_t>(m) * H + hd) * rp.Lmax + base) * kTN;
      if (part == 2) {
#pragma unroll
        for (int i = 0; i < NI; ++i) rp.vc[cache + tx + 16 * i] = v[i];
        continue;
      }
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        const int ih = tx + 16 * pr;
        const double cs = rp.cos_t[base * (kTN / 2) + ih], sn = rp.sin_t[base * (kTN / 2) + ih];
        const double a = static_cast<double>(v[pr]), bb = static_cast<double>(v[pr + 2]);
        const float o0 = __double2float_rn(__dsub_rn(__dmul_rn(a, cs), __dmul_rn(bb, sn)));
        const float o1 = __double2float_rn(__dadd_rn(__dmul_rn(a, sn), __dmul_rn(bb, cs)));
        float* dst = part == 0 ? rp.q + static_cast<size_t>(m) * rp.D + hd * kTN : rp.kc + cache;
        dst[ih] = o0;
        dst[ih + kTN / 2] = o1;
      }
    }
    return;
  }
  // accumulate: the residual update h += bitlinear(x) as one float add (bitnet.hpp:579-583); the
  // accumulated outputs are all requested before any is written
  float old[2][NI];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int m = m0 + ty + 16 * j, n = n0 + tx + 16 * i;
      old[j][i] = (accumulate && m < M && n < N) ? y[static_cast<size_t>(m) * N + n] : 0.0f;
    }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int m = m0 + ty + 16 * j;
    if (m >= M) continue;
    const double s = static_cast<double>(xscale[m]);
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      const int n = n0 + tx + 16 * i;
      if (n >= N) continue;
      const double v = __dmul_rn(__dmul_rn(static_cast<double>(acc[j][i]), static_cast<double>(alpha[n])), s);
      float* dst = y + static_cast<size_t>(m) * N + n;
      *dst = accumulate ? __fadd_rn(old[j][i], __double2float_rn(v)) : __double2float_rn(v);
    }
  }
}

// ---------------------------------------------------------------- tensor-core path (prefill)
// The same exact BitLinear on the 5th-generation tensor cores: tcgen05.mma kind::i8 (signed int8
// A and B from shared memory, int32 accumulation in TMEM — integer sums, so the result is the
// dp4a path's bit for bit).  One CTA = 128 tokens x 128 outputs; K in 128-byte blocks through a
// 2-stage ring, three CTAs per SM (66 KB of shared memory, 128 TMEM columns and <= 112 registers
// each), so the CTAs' epilogues run beside each other's mainloops (16384 x 3072 x 512 gate|up
// projection: one CTA per SM with 4 stages 212 us, two with 3 stages 151 us, three 114 us):
//   warp 0     TMA: the activation block (128 tokens x 128 int8, 128-byte swizzle);
//   warp 1     TMEM owner + MMA issuer: 4 MMAs (K = 32) per block, M = 128, N = 128;
//   warps 2-5  expand the weight block (128 rows x 128 two-bit codes, 4 KB packed) into int8 in
//              the 128-byte-swizzled K-major layout the MMA reads (thread = one output row, one
//              16-byte chunk per packed word, chunk index XOR row % 8), then, after the last block,
//              the epilogue: TMEM -> int32 -> y = float(double(acc) * alpha[n] * xscale[m])
//              (or y += that value), one row per thread.
constexpr int kTcM = 128, kTcN = 128, kTcKB = 128, kTcStages = 2, kTcThreads = 192;
constexpr int kTcStageA = kTcM * kTcKB, kTcStageB = kTcN * kTcKB;  // 16 KB each
constexpr int kTcSmem = kTcStages * (kTcStageA + kTcStageB) + 256 + 1024;

struct TernaryTcParams {
  const uint32_t* wp;
  const float* alpha;
  const float* xscale;
  float* y;
  int M, N, K, accumulate;
  int* status;
  int weights_early;  // decode path: no kernel still in the stream writes wp / alpha
};

__global__ void __launch_bounds__(kTcThreads, 3)
    ternary_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const TernaryTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kTcStages * kTcStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcStages * (kTcStageA + kTcStageB));
  uint64_t* a_full = bars;                 // [stages] TMA bytes
  uint64_t* b_full = a_full + kTcStages;   // [stages] 128 expanding threads
  uint64_t* empty = b_full + kTcStages;    // [stages] the stage's MMAs completed
  uint64_t* acc_full = empty + kTcStages;  // the last MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTcN, m0 = blockIdx.y * kTcM;
  const int nkb = p.K / kTcKB;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&b_full[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  griddep_wait();  // the activations come from the previous kernel (programmatic dependent launch)

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTcStages;
        if (kb >= kTcStages &&
            !mbar_wait(&empty[s], ((kb / kTcStages) - 1) & 1, abort_flag, p.status, kDevTimeoutProducer))
          break;
        mbar_arrive_expect_tx(&a_full[s], kTcStageA);
        tma_load_2d(sA + s * kTcStageA, &tmX, &a_full[s], kb * kTcKB, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kTcM, kTcN);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % kTcStages;
        const uint32_t par = (kb / kTcStages) & 1;
        ok = mbar_wait(&a_full[s], par, abort_flag, p.status, kDevTimeoutMma) &&
             mbar_wait(&b_full[s], par, abort_flag, p.status, kDevTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + s * kTcStageA), b_addr = smem_u32(sB + s * kTcStageB);
#pragma unroll
        for (int k = 0; k < kTcKB / 32; ++k)
          umma_i8_ss(tbase, sw128_desc(a_addr + k * 32, 16, 1024), sw128_desc(b_addr + k * 32, 16, 1024),
                     idesc, (kb != 0 || k != 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(acc_full);
    }
  } else {
    // warps 2..5: weight expansion, then the epilogue
    const int t = threadIdx.x - 64;          // 0..127: output row n0 + t during expansion
    const int n = n0 + t;
    const int wwords = p.K / 16;
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kTcStages;
      if (kb >= kTcStages &&
          !__all_sync(0xffffffffu, mbar_wait(&empty[s], ((kb / kTcStages) - 1) & 1, abort_flag,
                                            p.status, kDevTimeoutProducer))) {
        ok = false;
        break;
      }
      uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
      if (n < p.N) {
        const uint4* src = reinterpret_cast<const uint4*>(p.wp + static_cast<size_t>(n) * wwords + kb * 8);
        w0 = __ldg(src);
        w1 = __ldg(src + 1);
      }
      const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint8_t* row = sB + s * kTcStageB + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t wd = words[c];
        uint4 v;
        v.x = decode4(wd & 0xFFu);
        v.y = decode4((wd >> 8) & 0xFFu);
        v.z = decode4((wd >> 16) & 0xFFu);
        v.w = decode4(wd >> 24);
        *reinterpret_cast<uint4*>(row + ((c ^ (t & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();  // the generic-proxy writes are visible to the tensor core
      mbar_arrive(&b_full[s]);
    }
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = tokens m0 + 32 (w % 4) + lane; each
    // 32-column chunk's output scales are one coalesced load per warp, broadcast by shuffles, and
    // each 32 x 32 block of results goes through the warp's own shared-memory transpose so that
    // every store (and the read of an accumulated output) is one coalesced 128-byte row (the
    // ring's buffers are free after the last MMA; no barrier across warps)
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, p.status, kDevTimeoutEpilogue));
    float* s_tile = reinterpret_cast<float*>(sA) + (warp - 2) * 32 * 33;  // per warp [32][33]
    if (ok) {
      tc_fence_after();
      const int quad = warp & 3;
      const int mrow0 = m0 + quad * 32;
      const int m = mrow0 + lane;
      const double sx = m < p.M ? static_cast<double>(p.xscale[m]) : 0.0;
      const uint32_t taddr = tbase + (static_cast<uint32_t>(quad * 32) << 16);
      for (int c0 = 0; c0 < kTcN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + c0, r);
        const int nl = n0 + c0 + lane;
        const float a_lane = nl < p.N ? p.alpha[nl] : 0.0f;
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float aj = __shfl_sync(0xffffffffu, a_lane, j);
          const double v = __dmul_rn(__dmul_rn(static_cast<double>(static_cast<int>(r[j])),
                                               static_cast<double>(aj)), sx);
          s_tile[lane * 33 + j] = __double2float_rn(v);
        }
        __syncwarp();
        const int nn = n0 + c0 + lane;
        if (p.accumulate) {
          // the accumulated outputs are all requested before any is written (one round trip per
          // 16 rows instead of one per row)
#pragma unroll
          for (int r0 = 0; r0 < 32; r0 += 16) {
            float old[16];
#pragma unroll
            for (int rr = 0; rr < 16; ++rr) {
              const int mm = mrow0 + r0 + rr;
              old[rr] = (mm < p.M && nn < p.N) ? p.y[static_cast<size_t>(mm) * p.N + nn] : 0.0f;
            }
#pragma unroll
            for (int rr = 0; rr < 16; ++rr) {
              const int mm = mrow0 + r0 + rr;
              if (mm < p.M && nn < p.N)
                p.y[static_cast<size_t>(mm) * p.N + nn] = __fadd_rn(old[rr], s_tile[(r0 + rr) * 33 + lane]);
            }
          }
        } else {
          for (int rr = 0; rr < 32; ++rr) {
            const int mm = mrow0 + rr;
            if (mm < p.M && nn < p.N) p.y[static_cast<size_t>(mm) * p.N + nn] = s_tile[rr * 33 + lane];
          }
        }
        __syncwarp();
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kTcN);
  }
}

// ---------------------------------------------------------------- tensor-core path (decode)
// The same exact BitLinear for decode-sized inputs (fewer than tc_min_rows tokens, K <= 2048): one
// CTA = 128 tokens x TN outputs (TN = 32 or 64, so a decode projection spreads over 32-192 CTAs
// where 128-output tiles gave 8-48) with the CTA's whole expanded weight slice resident, so the
// only ring is the activations' (four 16 KB blocks: K <= 512 is resident at once).  The 128
// expanding threads fetch the CTA's packed weights and row scales, expand them into the
// 128-byte-swizzled K-major int8 layout and arrive on b_full — before waiting for the previous
// kernel when the caller states that no kernel still in the stream writes the weights (the LM's,
// packed when the model is created); warp 0 TMA-loads the activation blocks, warp 1 issues the
// K / 32 MMAs (M = 128, N = TN) into a TN-column TMEM accumulator, and the epilogue warps fetch
// the token scales and, for h +=, the accumulated outputs while the MMAs run.  The epilogue's
// operations are the prefill kernel's: y = float(double(acc) * alpha[n] * xscale[m]).  kRope (TN
// = 64: one head of q, k or v per tile): the q|k|v projection of one position per sequence, each
// thread rotating its token's RoPE pairs (c, c + 32) in double from the float outputs and
// writing q or the K / V cache row, as ternary_gemm_kernel<64, true> does.
constexpr int kTdKB = 128;     // k-block: 128 int8 = one 128-byte swizzled row
constexpr int kTdStages = 4;   // activation ring
constexpr int kTdMaxK = 2048;
constexpr int kTdThreads = 192;
constexpr int kTdStageA = kTcM * kTdKB;  // 16 KB
__host__ __device__ constexpr int td_smem_bytes(int TN, int K) {
  return kTdStages * kTdStageA + TN * K + TN * (K / 4) + TN * 4 + 256 + 1024;
}

static_assert(td_smem_bytes(64, kTdMaxK) <= 227 * 1024 && td_smem_bytes(32, kTdMaxK) <= 227 * 1024,
              "decode tile's shared memory at the largest K");
static_assert(td_smem_bytes(32, 4 * kTdKB) * 2 <= 228 * 1024 - 2 * 1024,
              "two 32-output CTAs per SM at K = 512");

template <int TN, bool kRope>
__global__ void __launch_bounds__(kTdThreads, 2)
    ternary_gemm_tcd_kernel(const __grid_constant__ CUtensorMap tmX, const TernaryTcParams p,
                            const RopeQkv rp) {
  static_assert(TN == 32 || TN == 64, "decode tile width");
  static_assert(!kRope || TN == 64, "a RoPE tile is one head");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int nkb = p.K / kTdKB;
  uint8_t* sA = smem;                                    // [kTdStages][128 x 128] int8, swizzled
  uint8_t* sB = sA + kTdStages * kTdStageA;              // [K / 128][TN x 128] int8, swizzled
  uint8_t* sRaw = sB + static_cast<size_t>(TN) * p.K;    // [TN][K / 4] packed codes
  float* sAlpha = reinterpret_cast<float*>(sRaw + TN * (p.K / 4));  // [TN]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sAlpha + TN);
  uint64_t* a_full = bars;                  // [kTdStages] TMA bytes
  uint64_t* empty = bars + kTdStages;       // [kTdStages] the block's MMAs completed
  uint64_t* b_full = bars + 2 * kTdStages;  // the 128 expanding threads
  uint64_t* acc_full = b_full + 1;          // the last MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t kCols = TN;  // a power of two >= 32

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TN, m0 = blockIdx.y * kTcM;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kTdStages; ++st) {
      mbar_init(&a_full[st], 1);
      mbar_init(&empty[st], 1);
    }
    mbar_init(b_full, 128);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      griddep_wait();  // the activations come from the previous kernel
      for (int kb = 0; kb < nkb; ++kb) {
        const int st = kb % kTdStages;
        if (kb >= kTdStages &&
            !mbar_wait(&empty[st], ((kb / kTdStages) - 1) & 1, abort_flag, p.status, kDevTimeoutProducer))
          break;
        mbar_arrive_expect_tx(&a_full[st], kTdStageA);
        tma_load_2d(sA + st * kTdStageA, &tmX, &a_full[st], kb * kTdKB, m0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(kTcM, TN);
      bool ok = mbar_wait(b_full, 0, abort_flag, p.status, kDevTimeoutMma);
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int st = kb % kTdStages;
        ok = mbar_wait(&a_full[st], (kb / kTdStages) & 1, abort_flag, p.status, kDevTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + st * kTdStageA);
        const uint32_t b_addr = smem_u32(sB + static_cast<size_t>(kb) * TN * kTdKB);
#pragma unroll
        for (int k = 0; k < kTdKB / 32; ++k)
          umma_i8_ss(tbase, sw128_desc(a_addr + k * 32, 16, 1024), sw128_desc(b_addr + k * 32, 16, 1024),
                     idesc, (kb != 0 || k != 0) ? 1u : 0u);
        umma_commit(&empty[st]);
      }
      if (ok) umma_commit(acc_full);
    }
  } else {
    // warps 2..5: the weights, then the epilogue
    const int t = threadIdx.x - 64;  // 0..127
    const int rowb = p.K / 4;        // packed bytes per output row
    if (!p.weights_early) griddep_wait();
    for (int q = t; q < TN * (rowb / 16); q += 128) {
      const int r = q / (rowb / 16), c = q - r * (rowb / 16);
      const bool in = n0 + r < p.N;
      const uint8_t* src = in ? reinterpret_cast<const uint8_t*>(p.wp) + static_cast<size_t>(n0 + r) * rowb + 16 * c
                              : reinterpret_cast<const uint8_t*>(p.wp);
      cp_async16(sRaw + r * rowb + 16 * c, src, in ? 16u : 0u);
    }
    cp_async_commit();
    if (t < TN) sAlpha[t] = n0 + t < p.N ? p.alpha[n0 + t] : 0.0f;
    cp_async_wait_all();
    asm volatile("bar.sync 1, 128;" ::: "memory");  // every packed row of the CTA has landed
    for (int q = t; q < TN * nkb; q += 128) {
      const int r = q % TN, kb = q / TN;
      const uint4* src = reinterpret_cast<const uint4*>(sRaw + r * rowb + kb * 32);
      const uint4 w0 = src[0], w1 = src[1];
      const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint8_t* row = sB + static_cast<size_t>(kb) * TN * kTdKB + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t wd = words[c];
        uint4 v;
        v.x = decode4(wd & 0xFFu);
        v.y = decode4((wd >> 8) & 0xFFu);
        v.z = decode4((wd >> 16) & 0xFFu);
        v.w = decode4(wd >> 24);
        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = v;
      }
    }
    fence_proxy_async_smem();  // the generic-proxy writes are visible to the tensor core
    mbar_arrive(b_full);
    if (p.weights_early) griddep_wait();  // the token scales and accumulated outputs are earlier kernels'
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = tokens m0 + 32 (w % 4) + lane
    const int quad = warp & 3;
    const int mrow0 = m0 + quad * 32;
    const int m = mrow0 + lane;
    const double sx = m < p.M ? static_cast<double>(p.xscale[m]) : 0.0;
    const uint32_t taddr = tbase + (static_cast<uint32_t>(quad * 32) << 16);
    if constexpr (kRope) {
      const int base = *rp.pos;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, p.status, kDevTimeoutEpilogue));
      if (ok) {
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(taddr, r0);
        tmem_ld_32x32b_x32(taddr + 32, r1);
        tmem_ld_wait();
        if (m < p.M) {
          float v[64];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __double2float_rn(__dmul_rn(
                __dmul_rn(static_cast<double>(static_cast<int>(r0[j])), static_cast<double>(sAlpha[j])), sx));
            v[32 + j] = __double2float_rn(__dmul_rn(
                __dmul_rn(static_cast<double>(static_cast<int>(r1[j])), static_cast<double>(sAlpha[32 + j])), sx));
          }
          const int part = n0 / rp.D, hd = (n0 % rp.D) / 64, H = rp.D / 64;
          const size_t cache = ((static_cast<size_t>(m) * H + hd) * rp.Lmax + base) * 64;
          float* dst = part == 0 ? rp.q + static_cast<size_t>(m) * rp.D + hd * 64
                                 : (part == 1 ? rp.kc : rp.vc) + cache;
          if (part != 2) {
            // RoPE (bitnet.hpp:472-488) of the pairs (ih, ih + 32), in double from the floats
#pragma unroll
            for (int ih = 0; ih < 32; ++ih) {
              const double cs = rp.cos_t[base * 32 + ih], sn = rp.sin_t[base * 32 + ih];
              const double a = static_cast<double>(v[ih]), bb = static_cast<double>(v[ih + 32]);
              v[ih] = __double2float_rn(__dsub_rn(__dmul_rn(a, cs), __dmul_rn(bb, sn)));
              v[ih + 32] = __double2float_rn(__dadd_rn(__dmul_rn(a, sn), __dmul_rn(bb, cs)));
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
    } else {
      // each 32 x 32 block leaves through the warp's own shared-memory transpose (coalesced rows)
      constexpr int NC = TN / 32;
      float old[NC][32];
      if (p.accumulate) {
        // the accumulated outputs, lane = column, requested while the MMAs run
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int nn = n0 + c * 32 + lane;
#pragma unroll
          for (int rr = 0; rr < 32; ++rr) {
            const int mm = mrow0 + rr;
            old[c][rr] = (mm < p.M && nn < p.N) ? p.y[static_cast<size_t>(mm) * p.N + nn] : 0.0f;
          }
        }
      }
      const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag, p.status, kDevTimeoutEpilogue));
      float* s_tile = reinterpret_cast<float*>(sA) + (warp - 2) * 32 * 33;  // per warp [32][33]
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(taddr + c * 32, r);
          const float a_lane = sAlpha[c * 32 + lane];
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float aj = __shfl_sync(0xffffffffu, a_lane, j);
            const double v = __dmul_rn(__dmul_rn(static_cast<double>(static_cast<int>(r[j])),
                                                 static_cast<double>(aj)), sx);
            s_tile[lane * 33 + j] = __double2float_rn(v);
          }
          __syncwarp();
          const int nn = n0 + c * 32 + lane;
#pragma unroll
          for (int rr = 0; rr < 32; ++rr) {
            const int mm = mrow0 + rr;
            if (mm < p.M && nn < p.N) {
              const float v = s_tile[rr * 33 + lane];
              p.y[static_cast<size_t>(mm) * p.N + nn] = p.accumulate ? __fadd_rn(old[c][rr], v) : v;
            }
          }
          __syncwarp();
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, kCols);
  }
}

// Launches the decode kernel on xq [M][K] (int8): the tensor map, the shared-memory limits once
// per device, and the grid (N / TN, M / 128).
template <int TN, bool kRope>
int launch_tcd(const TernaryTcParams& tp, const int8_t* xq, const RopeQkv& rp, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    DLM_CHECK_CUDA(cudaFuncSetAttribute(ternary_gemm_tcd_kernel<TN, kRope>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        td_smem_bytes(TN, kTdMaxK)));
    attr_set[dev] = true;
  }
  CUtensorMap tm;
  const uint64_t dims[2] = {static_cast<uint64_t>(tp.K), static_cast<uint64_t>(tp.M)};
  const uint64_t strides[1] = {static_cast<uint64_t>(tp.K)};
  const uint32_t box[2] = {kTdKB, kTcM};
  if (!encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B))
    return DLM_ERR_CUDA;
  DLM_CHECK_CUDA(launch_pdl(ternary_gemm_tcd_kernel<TN, kRope>, dim3(tp.N / TN, (tp.M + kTcM - 1) / kTcM),
      dim3(kTdThreads), td_smem_bytes(TN, tp.K), s, tm, tp, rp));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

}  // namespace

int ternary_pack(const float* w, int N, int K, uint32_t* packed, float* alpha, cudaStream_t s) {
  DLM_REQUIRE(w && packed && alpha, DLM_ERR_INVALID, "ternary_pack: null pointer");
  DLM_REQUIRE(N > 0 && K > 0 && K % 64 == 0, DLM_ERR_INVALID, "ternary_pack: K=%d must be a multiple of 64", K);
  ternary_pack_kernel<<<(N + 127) / 128, 128, 0, s>>>(w, N, K, packed, alpha);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int ternary_pack_per_tensor(const float* w, int N, int K, uint32_t* packed, float* alpha,
                            double* scratch, cudaStream_t s) {
  DLM_REQUIRE(w && packed && alpha && scratch, DLM_ERR_INVALID, "ternary_pack: null pointer");
  DLM_REQUIRE(N > 0 && K > 0 && K % 64 == 0, DLM_ERR_INVALID, "ternary_pack: K=%d must be a multiple of 64", K);
  tensor_absmean_kernel<<<1, 1, 0, s>>>(w, static_cast<size_t>(N) * K, scratch);
  DLM_CHECK_CUDA(cudaGetLastError());
  ternary_pack_alpha_kernel<<<(N + 127) / 128, 128, 0, s>>>(w, N, K, scratch, packed, alpha);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int quantize_act_i8(const float* x, int M, int K, int8_t* xq, float* xscale, cudaStream_t s) {
  DLM_REQUIRE(x && xq && xscale, DLM_ERR_INVALID, "quantize_act_i8: null pointer");
  DLM_REQUIRE(M > 0 && K > 0, DLM_ERR_INVALID, "quantize_act_i8: empty");
  const int warps = 8;
  DLM_CHECK_CUDA(launch_pdl(quant_act_kernel, dim3((M + warps - 1) / warps), dim3(warps * 32), 0, s,
      x, M, K, xq, xscale));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int ternary_gemm_i8(const uint32_t* wp, const float* alpha, const int8_t* xq, const float* xscale,
                    float* y, int M, int N, int K, cudaStream_t s, bool accumulate,
                    bool weights_resident) {
  DLM_REQUIRE(wp && alpha && xq && xscale && y, DLM_ERR_INVALID, "ternary_gemm_i8: null pointer");
  DLM_REQUIRE(K % 64 == 0 && K < (1 << 24), DLM_ERR_INVALID,
              "ternary_gemm_i8: K=%d must be a multiple of 64", K);
  DLM_REQUIRE((reinterpret_cast<uintptr_t>(wp) & 15) == 0 && (reinterpret_cast<uintptr_t>(xq) & 15) == 0,
              DLM_ERR_INVALID, "ternary_gemm_i8: packed weights / activations must be 16-byte aligned");
  if (M >= tc_min_rows() && K % kTcKB == 0 && N % 32 == 0) {
    // prefill-sized: the tensor-core path (same integer sums, same epilogue arithmetic)
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      DLM_CHECK_CUDA(cudaFuncSetAttribute(ternary_gemm_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem));
      attr_set[dev] = true;
    }
    CUtensorMap tm;
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K)};
    const uint32_t box[2] = {kTcKB, kTcM};
    if (!encode_tmap(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return DLM_ERR_CUDA;
    TernaryTcParams tp{wp, alpha, xscale, y, M, N, K, accumulate ? 1 : 0, device_status_ptr()};
    dim3 grid((N + kTcN - 1) / kTcN, (M + kTcM - 1) / kTcM);
    DLM_CHECK_CUDA(launch_pdl(ternary_gemm_tc_kernel, dim3(grid), dim3(kTcThreads), kTcSmem, s, tm,
        tp));
    DLM_CHECK_CUDA(cudaGetLastError());
    return DLM_OK;
  }
  if (tcd_enabled() && K % kTdKB == 0 && K <= kTdMaxK && N % 32 == 0) {
    // decode-sized: the tensor-core path with narrow tiles (same integer sums, same epilogue
    // arithmetic); 64-output tiles only where 32-output ones would need more than two CTAs per SM
    const TernaryTcParams tp{wp, alpha, xscale, y, M, N, K, accumulate ? 1 : 0, device_status_ptr(),
                             weights_resident ? 1 : 0};
    const long mt = (M + kTcM - 1) / kTcM;
    if (N % 64 != 0 || static_cast<long>(N / 32) * mt <= 2L * num_sms())
      return launch_tcd<32, false>(tp, xq, RopeQkv{}, s);
    return launch_tcd<64, false>(tp, xq, RopeQkv{}, s);
  }
  // 64-output tiles unless they leave more than half of the SMs idle (decode-sized projections)
  const long tiles64 = static_cast<long>((N + kTN - 1) / kTN) * ((M + kTM - 1) / kTM);
  if (2 * tiles64 < num_sms()) {
    dim3 grid((N + 31) / 32, (M + kTM - 1) / kTM);
    DLM_CHECK_CUDA(launch_pdl(ternary_gemm_kernel<32, false>, dim3(grid), dim3(kThreads), 0, s, wp, alpha,
        xq, xscale, y, M, N, K, accumulate ? 1 : 0, RopeQkv{}));
  } else {
    dim3 grid((N + kTN - 1) / kTN, (M + kTM - 1) / kTM);
    DLM_CHECK_CUDA(launch_pdl(ternary_gemm_kernel<kTN, false>, dim3(grid), dim3(kThreads), 0, s, wp, alpha,
        xq, xscale, y, M, N, K, accumulate ? 1 : 0, RopeQkv{}));
  }
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int ternary_tc_min_rows() { return tc_min_rows(); }

int ternary_gemm_qkv_rope(const uint32_t* wp, const float* alpha, const int8_t* xq,
                          const float* xscale, int M, int K, const RopeQkv& r, cudaStream_t s,
                          bool weights_resident) {
  DLM_REQUIRE(wp && alpha && xq && xscale && r.pos && r.cos_t && r.sin_t && r.q && r.kc && r.vc,
              DLM_ERR_INVALID, "ternary_gemm_qkv_rope: null pointer");
  DLM_REQUIRE(K % 64 == 0 && r.D % kTN == 0 && r.Lmax > 0, DLM_ERR_INVALID,
              "ternary_gemm_qkv_rope: K=%d, D=%d", K, r.D);
  DLM_REQUIRE((reinterpret_cast<uintptr_t>(wp) & 15) == 0 && (reinterpret_cast<uintptr_t>(xq) & 15) == 0,
              DLM_ERR_INVALID, "ternary_gemm_qkv_rope: packed weights / activations must be 16-byte aligned");
  const int N = 3 * r.D;
  if (tcd_enabled() && K % kTdKB == 0 && K <= kTdMaxK) {
    // the decode tensor-core path, one head per 64-output tile
    const TernaryTcParams tp{wp, alpha, xscale, nullptr, M, N, K, 0, device_status_ptr(),
                             weights_resident ? 1 : 0};
    return launch_tcd<64, true>(tp, xq, r, s);
  }
  dim3 grid(N / kTN, (M + kTM - 1) / kTM);
  DLM_CHECK_CUDA(launch_pdl(ternary_gemm_kernel<kTN, true>, dim3(grid), dim3(kThreads), 0, s, wp,
      alpha, xq, xscale, static_cast<float*>(nullptr), M, N, K, 0, r));
  return DLM_OK;
}

}  // namespace dlm

extern "C" {

int dlm_ternary_pack(const float* w, int N, int K, void* w_packed2b, float* row_scale, void* stream) {
  if (N == 0 || K == 0) return DLM_OK;
  return dlm::ternary_pack(w, N, K, static_cast<uint32_t*>(w_packed2b), row_scale,
                           static_cast<cudaStream_t>(stream));
}

int dlm_quantize_act_i8(const float* x, int M, int K, int8_t* xq, float* x_scale, void* stream) {
  if (M == 0 || K == 0) return DLM_OK;
  return dlm::quantize_act_i8(x, M, K, xq, x_scale, static_cast<cudaStream_t>(stream));
}

int dlm_ternary_gemm_i8(const void* w_packed2b, const float* row_scale, const int8_t* x,
                        const float* x_scale, float* y, int M, int N, int K, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  return dlm::ternary_gemm_i8(static_cast<const uint32_t*>(w_packed2b), row_scale, x, x_scale, y, M,
                              N, K, static_cast<cudaStream_t>(stream));
}

int dlm_bitlinear(const void* w_packed2b, const float* row_scale, const float* x, float* y, int M,
                  int N, int K, int8_t* xq_scratch, float* xscale_scratch, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = dlm::quantize_act_i8(x, M, K, xq_scratch, xscale_scratch, s);
  if (rc != DLM_OK) return rc;
  return dlm::ternary_gemm_i8(static_cast<const uint32_t*>(w_packed2b), row_scale, xq_scratch,
                              xscale_scratch, y, M, N, K, s);
}

}  // extern "C"
