// BitNet ternary tag LM on the GPU: batched prefill + greedy decode with a K/V cache.
//
// Replaces the LM around BitLinear that the reference runs on the host: BitNet::forward
// (src/models/bitnet.hpp:376-440: rms_norm :234, RoPE :472-488, causal attention :490-585, SwiGLU
// :589-617, tied lm_head :414-436) and the greedy rule of BitNetDenseInfer::generate
// (src/infer/bitnet.hpp:282-318), which re-runs the whole prefix for every new token.  Here the
// prompts of all sequences run as one prefill and every further token is one decode pass over a
// per-layer K/V cache; every position's arithmetic is the same as in the reference, so the cache
// changes no result.
//
// Numerics: the reference does its context arithmetic in double and rounds to float at fixed
// points; every kernel here performs the same double operations in the same order with explicit
// round-to-nearest intrinsics (no contraction), so the rms_norm outputs, RoPE (cos / sin tables
// computed on the host with the C library, as the reference does), attention scores and weighted
// sums, SwiGLU products and lm_head dots are bit-identical to the reference's.  The only functions
// whose last bit may differ are CUDA's double exp (softmax, SiLU) against the host C library's.  The
// BitLinear products are exact (int32 accumulation, double epilogue; ternary.cu).
//
// Layout: hidden state h [M, D] fp32 (M = B * S rows, row = sequence-major position); K/V cache
// [layer][b][head][pos][64] fp32 (K after RoPE); q|k|v, gate|up are each one GEMM.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "bitnet_lm.h"
#include "ptx.cuh"
#include "ternary.h"

namespace dlm {

namespace {

constexpr int kHeadDim = 64;
constexpr int kEos = 2;  // src/io/tokenizer.hpp:44

__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// p[0] + p[1] + ... + p[n-1] in index order from 0.0 (((0 + p0) + p1) + ...), by one thread: the
// reference's sequential sums.  The loads run eight elements ahead of the additions, so the
// dependent chain waits on the adder rather than on shared memory.
__device__ __forceinline__ double seq_sum(const double* p, int n) {
  double s = 0.0;
  const int n8 = n & ~7;
  int i = 0;
  if (n8 > 0) {
    double a[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = p[k];
    for (; i < n8; i += 8) {
      double b[8];
      const bool more = i + 8 < n8;
      if (more) {
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] = p[i + 8 + k];
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) s = __dadd_rn(s, a[k]);
      if (more) {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = b[k];
      }
    }
  }
  for (; i < n; ++i) s = __dadd_rn(s, p[i]);
  return s;
}

// One element of the absmax int8 quantization (quantize_activation_int8, bitnet.hpp:123-165).
__device__ __forceinline__ int8_t quant_one(float x, double scale, double inv) {
  int v = 0;
  if (scale != 0.0) {
    double r = round(__dmul_rn(static_cast<double>(x), inv));
    if (r > 127.0) r = 127.0;
    if (r < -127.0) r = -127.0;
    v = static_cast<int>(r);
  }
  return static_cast<int8_t>(v);
}

// Exact absmax int8 quantization of one row held in shared memory (quantize_activation_int8,
// bitnet.hpp:123-165), by one warp.
__device__ __forceinline__ void quant_row_warp(const float* row, int K, int8_t* q, float* scale_out) {
  const int lane = threadIdx.x & 31;
  double amax = 0.0;
  for (int i = lane; i < K; i += 32) amax = fmax(amax, fabs(static_cast<double>(row[i])));
  amax = warp_max_d(amax);
  const double scale = __ddiv_rn(amax, 127.0);
  const double inv = scale == 0.0 ? 0.0 : __ddiv_rn(1.0, scale);
  if (lane == 0) *scale_out = static_cast<float>(scale);
  for (int i = lane; i < K; i += 32) q[i] = quant_one(row[i], scale, inv);
}

// Row r of the output reads token tokens[b * ld_tok + base + p] (b = r / S, p = r % S, base =
// *pos_in or 0) and copies its embedding row.  Ids outside [0, vocab) use id 0 and raise *bad.
__global__ void embed_kernel(const int* __restrict__ tokens, int ld_tok, int S,
                             const int* __restrict__ pos_in, const float* __restrict__ embed, int V,
                             int D, float* __restrict__ h, int M, int* __restrict__ bad) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  const int r = blockIdx.x;
  if (r >= M) return;
  const int base = pos_in ? *pos_in : 0;
  int tok = tokens[static_cast<size_t>(r / S) * ld_tok + base + r % S];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0) atomicExch(bad, 1);
    tok = 0;
  }
  const float4* src = reinterpret_cast<const float4*>(embed + static_cast<size_t>(tok) * D);
  float4* dst = reinterpret_cast<float4*>(h + static_cast<size_t>(r) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = src[i];
}

// rms_norm (bitnet.hpp:234-250), one warp per output row: lane 0 adds the double squares of the
// row's elements in index order (as the reference's loop) — as fma(x, x, s), equal to
// s + x * x because the square of a float is exact in double — reading the row from shared
// memory 16 bytes at a time, eight elements ahead of the adds; then x * inv * w per element,
// rounded to float.  Output row r reads input row r * in_stride + in_off.  Optionally
// quantizes the normalised row (int8) and / or stores it transposed in double (out_t[d * ldt + r],
// the lm_head's operand layout; each thread writes the block's four rows of one element).
constexpr int kNormWarps = 4;
// per block: the rows as float
__host__ __device__ constexpr size_t norm_smem_bytes(int D) {
  return static_cast<size_t>(kNormWarps) * D * 4;
}
__global__ void __launch_bounds__(kNormWarps * 32)
    rms_norm_kernel(const float* __restrict__ h, int rows, int D, int in_stride, int in_off,
                    const float* __restrict__ w, double eps, int8_t* __restrict__ xq,
                    float* __restrict__ xs, double* __restrict__ out_t, int ldt) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  extern __shared__ __align__(16) float srow[];  // [kNormWarps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kNormWarps;
  const int r = r0 + warp;
  if (r >= rows && !out_t) return;  // (with out_t every warp reaches the block barrier below)
  float* row = srow + static_cast<size_t>(warp) * D;
  if (r < rows) {
    const float* src = h + (static_cast<size_t>(r) * in_stride + in_off) * D;
    for (int i = lane; i < D; i += 32) row[i] = src[i];
    __syncwarp();
    double inv = 0.0;
    if (lane == 0) {
      double ms = 0.0;
      int i = 0;
      if ((D & 7) == 0) {
        // rows of D floats start 16-byte aligned (D % 8 == 0, D * 4 bytes per row)
        const float4* p4 = reinterpret_cast<const float4*>(row);
        float4 a0 = p4[0], a1 = p4[1];
        for (; i < D; i += 8) {
          float4 b0 = a0, b1 = a1;
          if (i + 8 < D) {
            b0 = p4[(i >> 2) + 2];
            b1 = p4[(i >> 2) + 3];
          }
          const float e[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const double x = static_cast<double>(e[k]);
            ms = __fma_rn(x, x, ms);
          }
          a0 = b0;
          a1 = b1;
        }
      }
      for (; i < D; ++i) {
        const double x = static_cast<double>(row[i]);
        ms = __fma_rn(x, x, ms);
      }
      ms = __ddiv_rn(ms, static_cast<double>(D));
      inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(ms, eps)));
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int i = lane; i < D; i += 32)
      row[i] = __double2float_rn(
          __dmul_rn(__dmul_rn(static_cast<double>(row[i]), inv), static_cast<double>(w[i])));
    __syncwarp();
    if (xq) quant_row_warp(row, D, xq + static_cast<size_t>(r) * D, xs + r);
  }
  if (out_t) {
    __syncthreads();  // the block's normalised rows are in shared memory
    const int nr = min(kNormWarps, rows - r0);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      double* dst = out_t + static_cast<size_t>(d) * ldt + r0;
      for (int k = 0; k < nr; ++k) dst[k] = static_cast<double>(srow[static_cast<size_t>(k) * D + d]);
    }
  }
}

// RoPE (bitnet.hpp:472-488) on q and k of every head and append k, v to the cache.  Row r is
// sequence b = r / S at position base + r % S.  qkv [M, 3D] -> q [M, D]; cache [B][H][Lmax][64].
__global__ void rope_kv_kernel(const float* __restrict__ qkv, int M, int S, int D,
                               const int* __restrict__ pos_in, const double* __restrict__ cos_t,
                               const double* __restrict__ sin_t, float* __restrict__ q,
                               float* __restrict__ kc, float* __restrict__ vc, int Lmax) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  const int half = kHeadDim / 2;
  const int H = D / kHeadDim;
  const size_t total = static_cast<size_t>(M) * H * half;
  const int base = pos_in ? *pos_in : 0;
  for (size_t t = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(t % half);
    const int hd = static_cast<int>((t / half) % H);
    const int r = static_cast<int>(t / (static_cast<size_t>(half) * H));
    const int b = r / S, pos = base + r % S;
    const double cs = cos_t[pos * half + i], sn = sin_t[pos * half + i];
    const float* src = qkv + static_cast<size_t>(r) * 3 * D + hd * kHeadDim;
    auto rot = [&](const float* v, float* o0, float* o1) {
      const double a = static_cast<double>(v[i]), bb = static_cast<double>(v[i + half]);
      *o0 = __double2float_rn(__dsub_rn(__dmul_rn(a, cs), __dmul_rn(bb, sn)));
      *o1 = __double2float_rn(__dadd_rn(__dmul_rn(a, sn), __dmul_rn(bb, cs)));
    };
    float* qo = q + static_cast<size_t>(r) * D + hd * kHeadDim;
    rot(src, qo + i, qo + i + half);
    const size_t cache = ((static_cast<size_t>(b) * H + hd) * Lmax + pos) * kHeadDim;
    rot(src + D, kc + cache + i, kc + cache + i + half);
    vc[cache + i] = src[2 * D + i];
    vc[cache + i + half] = src[2 * D + i + half];
  }
}

// Causal attention (bitnet.hpp:536-569) of row r (sequence b, position pos) and one head over
// cache positions 0..pos: double scores in index order, exp, a sequential sum, then float
// accumulation of float(w_j * v_j) over j in order.  One block per (row, head).  For caches of up
// to kVStageMax positions the head's V rows 0..pos are first staged in shared memory with
// coalesced 16-byte loads (the output loop walks them in order, one dimension per thread); each
// thread's K row is loaded into registers as 16 independent 16-byte loads before its sequential
// dot product.
constexpr int kAttnThreads = 128;
constexpr int kVStageMax = 256;  // cache lengths up to which V is staged (64 KB of shared memory)
// cache lengths up to which K is staged as well, in rows of 68 floats (272 bytes: 16-byte aligned,
// and the 16-byte reads of eight consecutive rows fall in distinct banks); V then arrives in the
// same buffer once the scores are formed, so a block needs no more shared memory than for V alone
constexpr int kKStageMax = 128;
constexpr int kKRow = kHeadDim + 4;
// doubles before the staged V rows, rounded up to an even count so that V starts 16-byte aligned
// (its rows are written with 16-byte stores) whatever the cache length
__host__ __device__ constexpr int attn_head_doubles(int Lmax) { return (kHeadDim + Lmax + 40 + 1) & ~1; }
__host__ __device__ constexpr size_t attn_smem_bytes(int Lmax) {
  return attn_head_doubles(Lmax) * sizeof(double) +
         (Lmax <= kKStageMax ? static_cast<size_t>(Lmax) * kKRow * 4
          : Lmax <= kVStageMax ? static_cast<size_t>(Lmax) * kHeadDim * 4 : 0);
}
__global__ void __launch_bounds__(kAttnThreads)
    attention_kernel(const float* __restrict__ q, int M, int S, int D, const int* __restrict__ pos_in,
                     const float* __restrict__ kc, const float* __restrict__ vc, int Lmax,
                     float* __restrict__ out) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  extern __shared__ double sh[];  // [64] q, [Lmax] scores, [40] reduction, then K rows / V rows (f32)
  double* sq = sh;
  double* ss = sh + kHeadDim;
  double* red = ss + Lmax;
  float* sv = reinterpret_cast<float*>(sh + attn_head_doubles(Lmax));
  const int H = D / kHeadDim;
  const int r = blockIdx.x / H, hd = blockIdx.x % H;
  if (r >= M) return;
  const int b = r / S, pos = (pos_in ? *pos_in : 0) + r % S;
  const int n = pos + 1;
  const float* qr = q + static_cast<size_t>(r) * D + hd * kHeadDim;
  const float* kb = kc + (static_cast<size_t>(b) * H + hd) * Lmax * kHeadDim;
  const float* vb = vc + (static_cast<size_t>(b) * H + hd) * Lmax * kHeadDim;
  for (int d = threadIdx.x; d < kHeadDim; d += blockDim.x) sq[d] = static_cast<double>(qr[d]);
  const bool staged = Lmax <= kVStageMax;
  const bool kstaged = Lmax <= kKStageMax;
  float* skk = sv;  // K rows (kstaged), then V in the same buffer
  if (kstaged) {
    // K rows 0..n-1 by coalesced asynchronous 16-byte copies (read per thread from the global
    // cache instead, each 16-byte load of a warp touches 32 rows); 16-byte aligned:
    // attn_head_doubles is even
    for (int i = threadIdx.x; i < n * (kHeadDim / 4); i += blockDim.x)
      cp_async16(skk + (i >> 4) * kKRow + 4 * (i & 15), kb + 4 * i, 16);
    cp_async_commit();
    cp_async_wait_all();
  } else if (staged) {
    // V rows 0..n-1 into shared memory by asynchronous 16-byte copies, all in flight at once:
    // they land while the scores are formed
    for (int i = threadIdx.x; i < n * (kHeadDim / 4); i += blockDim.x)
      cp_async16(sv + 4 * i, vb + 4 * i, 16);
    cp_async_commit();
  }
  const float* vrows = staged ? sv : vb;
  __syncthreads();
  double mx = -1e300;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float4* kj = kstaged ? reinterpret_cast<const float4*>(skk + static_cast<size_t>(j) * kKRow)
                               : reinterpret_cast<const float4*>(kb + static_cast<size_t>(j) * kHeadDim);
    float4 kr[kHeadDim / 4];
#pragma unroll
    for (int i = 0; i < kHeadDim / 4; ++i) kr[i] = kj[i];
    const float* kf = reinterpret_cast<const float*>(kr);
    double dot = 0.0;
#pragma unroll
    // fma equals the multiply-then-add: q and k are floats, whose product is exact in double
    for (int d = 0; d < kHeadDim; ++d) dot = __fma_rn(sq[d], static_cast<double>(kf[d]), dot);
    dot = __dmul_rn(dot, 0.125);  // 1 / sqrt(64), exact
    ss[j] = dot;
    mx = fmax(mx, dot);
  }
  mx = warp_max_d(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (kstaged) {
    // every thread has its score: V rows 0..n-1 into the K buffer, landing during the
    // exponentials and the sequential sum
    for (int i = threadIdx.x; i < n * (kHeadDim / 4); i += blockDim.x)
      cp_async16(sv + 4 * i, vb + 4 * i, 16);
    cp_async_commit();
  }
  if (threadIdx.x == 0) {
    double m = red[0];
    for (int w = 1; w < kAttnThreads / 32; ++w) m = fmax(m, red[w]);
    red[kAttnThreads / 32] = m;
  }
  __syncthreads();
  mx = red[kAttnThreads / 32];
  for (int j = threadIdx.x; j < n; j += blockDim.x) ss[j] = exp(__dsub_rn(ss[j], mx));
  __syncthreads();
  if (threadIdx.x == 0) red[kAttnThreads / 32 + 1] = __ddiv_rn(1.0, seq_sum(ss, n));
  __syncthreads();
  const double inv = red[kAttnThreads / 32 + 1];
  // the weights w_j = e_j / sum, once per key
  for (int j = threadIdx.x; j < n; j += blockDim.x) ss[j] = __dmul_rn(ss[j], inv);
  if (staged) cp_async_wait_all();  // this thread's V copies have landed
  __syncthreads();
  for (int d = threadIdx.x; d < kHeadDim; d += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < n; ++j)
      acc = __fadd_rn(acc, __double2float_rn(__dmul_rn(ss[j], static_cast<double>(vrows[j * kHeadDim + d]))));
    out[static_cast<size_t>(r) * D + hd * kHeadDim + d] = acc;
  }
}

// The same causal attention for a prefill of S > 1 positions per sequence: one block per
// (sequence, head) stages the head's K and V rows 0..base+S-1 in shared memory once, and each warp
// takes query rows in turn (row = one position): lanes compute the double scores of keys lane,
// lane + 32, ... (each a sequential 64-term sum in index order), the row max by shuffles, the
// exponentials, lane 0 the sequential sum of the weights, and each lane two output dimensions,
// accumulated in float over j in order — the reference's operation order for every value.
constexpr int kAttnSeqWarps = 8;
constexpr int kAttnSeqMax = 128;  // staged positions (K and V: 64 KB)
// K rows are staged with a stride of 65 floats, so the 32 lanes' keys at one dimension fall in 32
// different banks; the float count of the K block is rounded up to a multiple of four, so V
// (written with 16-byte stores) and the doubles after it stay 16-byte aligned for any n.
constexpr int kKStride = kHeadDim + 1;
__host__ __device__ constexpr size_t attn_seq_k_floats(int n) {
  return (static_cast<size_t>(n) * kKStride + 3) & ~static_cast<size_t>(3);
}
__host__ __device__ constexpr size_t attn_seq_smem_bytes(int n) {
  return (attn_seq_k_floats(n) + static_cast<size_t>(n) * kHeadDim) * 4 +
         kAttnSeqWarps * (kHeadDim + n) * sizeof(double);
}
__global__ void __launch_bounds__(kAttnSeqWarps * 32)
    attention_seq_kernel(const float* __restrict__ q, int S, int D, const int* __restrict__ pos_in,
                         const float* __restrict__ kc, const float* __restrict__ vc, int Lmax,
                         float* __restrict__ out) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  extern __shared__ __align__(16) double shd[];
  const int H = D / kHeadDim;
  const int b = blockIdx.x / H, hd = blockIdx.x % H;
  const int base = pos_in ? *pos_in : 0;
  const int nmax = base + S;  // positions any row of this block attends to
  float* sk = reinterpret_cast<float*>(shd);
  float* sv = sk + attn_seq_k_floats(nmax);
  double* wbuf = reinterpret_cast<double*>(sv + static_cast<size_t>(nmax) * kHeadDim);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double* sq = wbuf + static_cast<size_t>(warp) * (kHeadDim + nmax);
  double* ss = sq + kHeadDim;
  {
    const size_t head = (static_cast<size_t>(b) * H + hd) * Lmax * kHeadDim;
    const float4* ks = reinterpret_cast<const float4*>(kc + head);
    const float4* vs = reinterpret_cast<const float4*>(vc + head);
    float4* vd = reinterpret_cast<float4*>(sv);
    for (int i = threadIdx.x; i < nmax * (kHeadDim / 4); i += blockDim.x) {
      const float4 kv = ks[i];
      float* kd = sk + (i >> 4) * kKStride + (i & 15) * 4;
      kd[0] = kv.x;
      kd[1] = kv.y;
      kd[2] = kv.z;
      kd[3] = kv.w;
      vd[i] = vs[i];
    }
  }
  __syncthreads();
  for (int p = warp; p < S; p += kAttnSeqWarps) {
    const int r = b * S + p;
    const int n = base + p + 1;
    const float* qr = q + static_cast<size_t>(r) * D + hd * kHeadDim;
    sq[lane] = static_cast<double>(qr[lane]);
    sq[lane + 32] = static_cast<double>(qr[lane + 32]);
    __syncwarp();
    double mx = -1e300;
    for (int j = lane; j < n; j += 32) {
      const float* kj = sk + static_cast<size_t>(j) * kKStride;
      double dot = 0.0;
#pragma unroll 16
      // fma equals the multiply-then-add: q and k are floats, whose product is exact in double
      for (int d = 0; d < kHeadDim; ++d) dot = __fma_rn(sq[d], static_cast<double>(kj[d]), dot);
      dot = __dmul_rn(dot, 0.125);  // 1 / sqrt(64), exact
      ss[j] = dot;
      mx = fmax(mx, dot);
    }
    mx = warp_max_d(mx);
    for (int j = lane; j < n; j += 32) ss[j] = exp(__dsub_rn(ss[j], mx));
    __syncwarp();
    double inv = 0.0;
    if (lane == 0) inv = __ddiv_rn(1.0, seq_sum(ss, n));
    inv = __shfl_sync(0xffffffffu, inv, 0);
    // the weights w_j = e_j / sum, once per key
    for (int j = lane; j < n; j += 32) ss[j] = __dmul_rn(ss[j], inv);
    __syncwarp();
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int j = 0; j < n; ++j) {
      const double wj = ss[j];
      const float* vj = sv + static_cast<size_t>(j) * kHeadDim;
      acc0 = __fadd_rn(acc0, __double2float_rn(__dmul_rn(wj, static_cast<double>(vj[lane]))));
      acc1 = __fadd_rn(acc1, __double2float_rn(__dmul_rn(wj, static_cast<double>(vj[lane + 32]))));
    }
    float* orow = out + static_cast<size_t>(r) * D + hd * kHeadDim;
    orow[lane] = acc0;
    orow[lane + 32] = acc1;
    __syncwarp();  // ss / sq are rewritten by this warp's next row
  }
}

// SwiGLU (bitnet.hpp:603-610) of gate|up [M, 2F] -> float(silu(g) * u), then int8 quantization;
// one block per row: every thread computes its elements and their absolute maximum, the block
// combines the maxima, and every thread quantizes its own elements (a maximum and per-element
// operations, so the same bits in any split).  kSwiThreads = 512 for decode-sized inputs (three
// of F = 1536 elements per thread: fewer dependent double exp / divide chains per thread, 9.7 ->
// 7.7 µs for 256 rows) and 256 for prefill-sized ones (16384 rows: 1247 µs against 1717 µs with
// 512, where the blocks already fill the SMs).
constexpr int kSwiRowsWide = 1024;  // rows below which a row gets 512 threads
template <int kSwiThreads>
__global__ void __launch_bounds__(kSwiThreads)
    swiglu_quant_kernel(const float* __restrict__ gu, int M, int F, int8_t* __restrict__ xq,
                        float* __restrict__ xs) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  extern __shared__ float srow[];  // [F]
  __shared__ double s_amax[kSwiThreads / 32];
  const int r = blockIdx.x;
  if (r >= M) return;
  const float* g = gu + static_cast<size_t>(r) * 2 * F;
  double amax = 0.0;
  for (int f = threadIdx.x; f < F; f += kSwiThreads) {
    const double gv = static_cast<double>(g[f]);
    const double silu = __ddiv_rn(gv, __dadd_rn(1.0, exp(-gv)));
    const float v = __double2float_rn(__dmul_rn(silu, static_cast<double>(g[F + f])));
    srow[f] = v;
    amax = fmax(amax, fabs(static_cast<double>(v)));
  }
  amax = warp_max_d(amax);
  if ((threadIdx.x & 31) == 0) s_amax[threadIdx.x >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kSwiThreads / 32; ++w) amax = fmax(amax, s_amax[w]);
  const double scale = __ddiv_rn(amax, 127.0);
  const double inv = scale == 0.0 ? 0.0 : __ddiv_rn(1.0, scale);
  if (threadIdx.x == 0) xs[r] = static_cast<float>(scale);
  int8_t* q = xq + static_cast<size_t>(r) * F;
  for (int f = threadIdx.x; f < F; f += kSwiThreads) q[f] = quant_one(srow[f], scale, inv);
}

// Tied lm_head (bitnet.hpp:414-436): logits[r, v] = float(sum_d double(x[r, d]) * double(E[v, d]))
// with d in increasing order for every output (the products are exact in double, so fma equals
// the reference's multiply-then-add).  Both operands are read already in double and transposed —
// xT [D][ldx] (written by the final rms_norm) and ET [D][ldv] (the embedding, transposed once when
// the model is created, zero beyond V) — so K chunks of 16 arrive by asynchronous 16-byte copies
// straight into the tiles the loop reads, double-buffered (converting fp32 chunks in every block
// instead repeated each x element's conversion for all 250 vocabulary tiles).  Tile: 64 rows x 64
// vocab ids; each thread owns 4 rows (two adjacent pairs, each read by one 16-byte load that the
// warp's 16 threads of a row pair share) x 4 ids (the L1 data pipe bounds it: 84 % of its
// wavefronts against 54 % of the fp64 pipe, measured on one launch).  ldx and ldv are multiples
// of 64, so every copy is in bounds (rows r >= R are computed and not stored).
constexpr int kLmR = 64, kLmV = 64, kLmK = 16;
__global__ void __launch_bounds__(256)
    lm_head_kernel(const double* __restrict__ xT, int ldx, int R, int D,
                   const double* __restrict__ ET, int ldv, int V, float* __restrict__ logits) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  __shared__ __align__(16) double xs[2][kLmK][kLmR];
  __shared__ __align__(16) double es[2][kLmK][kLmV];
  const int r0 = blockIdx.y * kLmR, v0 = blockIdx.x * kLmV;
  // v = v0 + tx + 16 i;  r = r0 + 2 ty + 32 (j >> 1) + (j & 1)
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  double acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.0;
  // chunk k0 into buffer b: per tile row kk, 32 copies of two doubles (x then E)
  auto fetch = [&](int k0, int b) {
#pragma unroll
    for (int t = threadIdx.x; t < kLmK * (kLmR + kLmV) / 2; t += 256) {
      const int kk = t / ((kLmR + kLmV) / 2), q = t % ((kLmR + kLmV) / 2);
      if (q < kLmR / 2)
        cp_async16(&xs[b][kk][2 * q], xT + static_cast<size_t>(k0 + kk) * ldx + r0 + 2 * q, 16);
      else
        cp_async16(&es[b][kk][2 * (q - kLmR / 2)],
                   ET + static_cast<size_t>(k0 + kk) * ldv + v0 + 2 * (q - kLmR / 2), 16);
    }
    cp_async_commit();
  };
  fetch(0, 0);
  int b = 0;
  for (int k0 = 0; k0 < D; k0 += kLmK, b ^= 1) {
    if (k0 + kLmK < D) {
      fetch(k0 + kLmK, b ^ 1);  // its buffer was last read before the previous closing barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      cp_async_wait_all();
    }
    __syncthreads();  // chunk k0 landed for every thread
#pragma unroll 4
    for (int kk = 0; kk < kLmK; ++kk) {
      double xv[4], ev[4];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const double2 p = *reinterpret_cast<const double2*>(&xs[b][kk][2 * ty + 32 * jj]);
        xv[2 * jj] = p.x;
        xv[2 * jj + 1] = p.y;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) ev[i] = es[b][kk][tx + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = __fma_rn(xv[j], ev[i], acc[j][i]);
    }
    __syncthreads();  // every thread is done with buffer b
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = r0 + 2 * ty + 32 * (j >> 1) + (j & 1);
    if (r >= R) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = v0 + tx + 16 * i;
      if (v < V) logits[static_cast<size_t>(r) * V + v] = __double2float_rn(acc[j][i]);
    }
  }
}

// Embedding E [V][D] (fp32) -> ET [D][ldv] (double), zero for v in [V, ldv): the lm_head's operand.
__global__ void embed_transpose_kernel(const float* __restrict__ E, int V, int D, int ldv,
                                       double* __restrict__ ET) {
  __shared__ float tile[32][33];
  const int v0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int v = v0 + k, d = d0 + threadIdx.x;
    tile[k][threadIdx.x] = (v < V && d < D) ? E[static_cast<size_t>(v) * D + d] : 0.0f;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int d = d0 + k, v = v0 + threadIdx.x;
    if (d < D && v < ldv) ET[static_cast<size_t>(d) * ldv + v] = static_cast<double>(tile[threadIdx.x][k]);
  }
}

// Greedy step (src/infer/bitnet.hpp:290-318) for sequence b = blockIdx.x: argmax of logits[b]
// (ties to the smallest id).  The logits belong to position pos = *pos_io; a live sequence whose
// argmax is <eos> stops, otherwise the id is appended at position pos + 1 and to out[b].  A stopped
// sequence is fed <eos> so the batch keeps a uniform shape (its outputs are never read).
__global__ void __launch_bounds__(256)
    greedy_kernel(const float* __restrict__ logits, int V, const int* __restrict__ pos_io, int P,
                  int* __restrict__ tokens, int ld_tok, int* __restrict__ done,
                  int* __restrict__ out, int ld_out, int* __restrict__ out_len) {
  griddep_wait();  // inputs come from the previous kernel (programmatic dependent launch)
  __shared__ float bv[8];
  __shared__ int bi[8];
  const int b = blockIdx.x;
  const float* row = logits + static_cast<size_t>(b) * V;
  // the largest logit, the lowest id among equal ones (a NaN is never taken): an order-free rule,
  // so any split of the row gives the same id.  16-byte loads, four in flight per thread.
  float best = -INFINITY;
  int idx = 0x7fffffff;
  auto take = [&](float x, int v) {
    if (x > best || (x == best && v < idx)) {
      best = x;
      idx = v;
    }
  };
  const int V4 = (V & 3) == 0 ? V / 4 : 0;  // rows 16-byte aligned when V % 4 == 0
  const float4* row4 = reinterpret_cast<const float4*>(row);
  int q = threadIdx.x;
  for (; q + 3 * 256 < V4; q += 4 * 256) {
    float4 c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = row4[q + u * 256];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = 4 * (q + u * 256);
      take(c[u].x, v);
      take(c[u].y, v + 1);
      take(c[u].z, v + 2);
      take(c[u].w, v + 3);
    }
  }
  for (; q < V4; q += 256) {
    const float4 c = row4[q];
    take(c.x, 4 * q);
    take(c.y, 4 * q + 1);
    take(c.z, 4 * q + 2);
    take(c.w, 4 * q + 3);
  }
  for (int v = 4 * V4 + threadIdx.x; v < V; v += 256) take(row[v], v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    take(ob, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) take(bv[w], bi[w]);
    bi[0] = idx;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int pos = *pos_io;
  const int step = pos - (P - 1);
  int next = kEos;
  if (!done[b]) {
    const int t = bi[0] == 0x7fffffff ? 0 : bi[0];
    if (t == kEos) {
      done[b] = 1;
    } else {
      out[static_cast<size_t>(b) * ld_out + step] = t;
      out_len[b] = step + 1;
      next = t;
    }
  }
  if (pos + 1 < ld_tok) tokens[static_cast<size_t>(b) * ld_tok + pos + 1] = next;
}

__global__ void set_int_kernel(int* p, int v) {
  griddep_wait();
  *p = v;
}
__global__ void inc_int_kernel(int* p) {
  griddep_wait();
  *p += 1;
}

int grid1d(size_t n, int t) {
  size_t g = (n + t - 1) / t;
  return static_cast<int>(g < 65535 * 16 ? g : 65535 * 16);
}

}  // namespace

// ================================================================== model

std::vector<BitNetWeightSpec> bitnet_weight_specs(const BitNetCfg& c) {
  std::vector<BitNetWeightSpec> S;
  const int64_t D = c.d_model, F = c.ffn_dim;
  S.push_back({"embed", {c.vocab, D}});
  S.push_back({"final_norm", {D}});
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    S.push_back({p + "attn_norm", {D}});
    S.push_back({p + "wq", {D, D}});
    S.push_back({p + "wk", {D, D}});
    S.push_back({p + "wv", {D, D}});
    S.push_back({p + "wo", {D, D}});
    S.push_back({p + "ffn_norm", {D}});
    S.push_back({p + "w_gate", {F, D}});
    S.push_back({p + "w_up", {F, D}});
    S.push_back({p + "w_down", {D, F}});
  }
  return S;
}

int bitnet_check_cfg(const BitNetCfg& c) {
  DLM_REQUIRE(c.vocab > 0 && c.n_layers > 0 && c.max_seq > 0 && c.max_seq <= 4096, DLM_ERR_INVALID,
              "bitnet: vocab / layers / max_seq out of range");
  DLM_REQUIRE(c.d_model > 0 && c.d_model % 64 == 0 && c.d_model <= 4096 &&
                  c.n_heads * kHeadDim == c.d_model,
              DLM_ERR_INVALID, "bitnet: d_model must be 64 * n_heads (head_dim 64) and <= 4096");
  DLM_REQUIRE(c.ffn_dim > 0 && c.ffn_dim % 64 == 0 && c.ffn_dim <= 8192, DLM_ERR_INVALID,
              "bitnet: ffn_dim must be a multiple of 64 and <= 8192");
  DLM_REQUIRE(c.rms_eps > 0.0 && c.rope_base > 0.0, DLM_ERR_INVALID, "bitnet: bad eps / rope base");
  return DLM_OK;
}

BitNetLM::~BitNetLM() {
  release_plan();
  for (void* p : wallocs_) cudaFree(p);
}

void BitNetLM::release_plan() {
  if (step_graph_) cudaGraphExecDestroy(step_graph_);
  step_graph_ = nullptr;
  if (cap_stream_) cudaStreamDestroy(cap_stream_);
  cap_stream_ = nullptr;
  if (abuf_) cudaFree(abuf_);
  abuf_ = nullptr;
  B_ = P_ = L_ = 0;
}

template <typename T>
T* BitNetLM::walloc(size_t n) {
  void* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  wallocs_.push_back(p);
  return static_cast<T*>(p);
}

int BitNetLM::create(const BitNetCfg& cfg, int n, const char* const* names, const float* const* ptrs,
                     const int64_t* numels, cudaStream_t s) {
  int rc = bitnet_check_cfg(cfg);
  if (rc != DLM_OK) return rc;
  cfg_ = cfg;
  std::unordered_map<std::string, std::pair<const float*, int64_t>> given;
  for (int i = 0; i < n; ++i) {
    DLM_REQUIRE(names[i] != nullptr && ptrs[i] != nullptr, DLM_ERR_INVALID,
                "bitnet_create: null name or pointer at %d", i);
    given[names[i]] = {ptrs[i], numels ? numels[i] : -1};
  }
  // every source tensor the packing kernels read must be device memory: host arrays are staged
  std::vector<void*> staged;
  auto on_device = [&](const float* p, size_t elems, const float** out) -> int {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) == cudaSuccess &&
        (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged)) {
      *out = p;
      return DLM_OK;
    }
    cudaGetLastError();
    void* d = nullptr;
    DLM_CHECK_CUDA(cudaMalloc(&d, elems * sizeof(float)));
    staged.push_back(d);
    DLM_CHECK_CUDA(cudaMemcpy(d, p, elems * sizeof(float), cudaMemcpyHostToDevice));
    *out = static_cast<const float*>(d);
    return DLM_OK;
  };
  struct StageFree {
    std::vector<void*>* v;
    cudaStream_t s;
    ~StageFree() {
      cudaStreamSynchronize(s);
      for (void* p : *v) cudaFree(p);
    }
  } stage_free{&staged, s};
  std::unordered_map<std::string, const float*> src;
  for (const auto& sp : bitnet_weight_specs(cfg)) {
    auto it = given.find(sp.name);
    DLM_REQUIRE(it != given.end(), DLM_ERR_NOT_FOUND, "bitnet_create: missing weight %s", sp.name.c_str());
    int64_t ne = 1;
    for (auto d : sp.shape) ne *= d;
    DLM_REQUIRE(it->second.second < 0 || it->second.second == ne, DLM_ERR_INVALID,
                "bitnet_create: %s has %lld elements, expected %lld", sp.name.c_str(),
                static_cast<long long>(it->second.second), static_cast<long long>(ne));
    const float* d = nullptr;
    rc = on_device(it->second.first, static_cast<size_t>(ne), &d);
    if (rc != DLM_OK) return rc;
    src[sp.name] = d;
  }
  const int D = cfg.d_model, F = cfg.ffn_dim, V = cfg.vocab;
  auto copy = [&](const float* from, size_t elems) -> float* {
    float* d = walloc<float>(elems);
    if (!d || cudaMemcpyAsync(d, from, elems * 4, cudaMemcpyDefault, s) != cudaSuccess) return nullptr;
    return d;
  };
  embed_ = copy(src["embed"], static_cast<size_t>(V) * D);
  final_norm_ = copy(src["final_norm"], D);
  DLM_REQUIRE(embed_ && final_norm_, DLM_ERR_NOMEM, "bitnet_create: out of device memory");
  DLM_REQUIRE(D % kLmK == 0, DLM_ERR_INVALID, "bitnet_create: d_model %d must be a multiple of %d", D,
              kLmK);
  // the lm_head's operand: the embedding transposed to [D][ldv] in double
  ldv_ = (V + kLmV - 1) / kLmV * kLmV;
  embT_ = walloc<double>(static_cast<size_t>(D) * ldv_);
  DLM_REQUIRE(embT_, DLM_ERR_NOMEM, "bitnet_create: out of device memory");
  embed_transpose_kernel<<<dim3((ldv_ + 31) / 32, (D + 31) / 32), dim3(32, 8), 0, s>>>(embed_, V, D,
                                                                                    ldv_, embT_);
  DLM_CHECK_CUDA(cudaGetLastError());
  double* scratch = walloc<double>(1);
  DLM_REQUIRE(scratch, DLM_ERR_NOMEM, "bitnet_create: out of device memory");
  // pack rows [row0, row0 + N) of a concatenated linear from one source tensor
  auto pack = [&](const float* w, int N, int K, uint32_t* packed, float* alpha) -> int {
    if (cfg.per_tensor_scale) return ternary_pack_per_tensor(w, N, K, packed, alpha, scratch, s);
    return ternary_pack(w, N, K, packed, alpha, s);
  };
  layers_.resize(cfg.n_layers);
  for (int l = 0; l < cfg.n_layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    Layer& L = layers_[l];
    L.attn_norm = copy(src[p + "attn_norm"], D);
    L.ffn_norm = copy(src[p + "ffn_norm"], D);
    L.wqkv = walloc<uint32_t>(static_cast<size_t>(3 * D) * D / 16);
    L.aqkv = walloc<float>(3 * D);
    L.wo = walloc<uint32_t>(static_cast<size_t>(D) * D / 16);
    L.ao = walloc<float>(D);
    L.wgu = walloc<uint32_t>(static_cast<size_t>(2 * F) * D / 16);
    L.agu = walloc<float>(2 * F);
    L.wd = walloc<uint32_t>(static_cast<size_t>(D) * F / 16);
    L.ad = walloc<float>(D);
    DLM_REQUIRE(L.attn_norm && L.ffn_norm && L.wqkv && L.aqkv && L.wo && L.ao && L.wgu && L.agu &&
                    L.wd && L.ad,
                DLM_ERR_NOMEM, "bitnet_create: out of device memory");
    const size_t dd = static_cast<size_t>(D) * D / 16;
    if ((rc = pack(src[p + "wq"], D, D, L.wqkv, L.aqkv)) != DLM_OK) return rc;
    if ((rc = pack(src[p + "wk"], D, D, L.wqkv + dd, L.aqkv + D)) != DLM_OK) return rc;
    if ((rc = pack(src[p + "wv"], D, D, L.wqkv + 2 * dd, L.aqkv + 2 * D)) != DLM_OK) return rc;
    if ((rc = pack(src[p + "wo"], D, D, L.wo, L.ao)) != DLM_OK) return rc;
    if ((rc = pack(src[p + "w_gate"], F, D, L.wgu, L.agu)) != DLM_OK) return rc;
    if ((rc = pack(src[p + "w_up"], F, D, L.wgu + static_cast<size_t>(F) * D / 16, L.agu + F)) != DLM_OK)
      return rc;
    if ((rc = pack(src[p + "w_down"], D, F, L.wd, L.ad)) != DLM_OK) return rc;
  }
  // RoPE tables with the host C library (the reference's own cos / sin / pow, bitnet.hpp:476-481)
  const int half = kHeadDim / 2;
  std::vector<double> ct(static_cast<size_t>(cfg.max_seq) * half), st(ct.size());
  for (int pos = 0; pos < cfg.max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const double freq = 1.0 / std::pow(cfg.rope_base, static_cast<double>(2 * i) / static_cast<double>(kHeadDim));
      const double angle = static_cast<double>(pos) * freq;
      ct[static_cast<size_t>(pos) * half + i] = std::cos(angle);
      st[static_cast<size_t>(pos) * half + i] = std::sin(angle);
    }
  cos_t_ = walloc<double>(ct.size());
  sin_t_ = walloc<double>(st.size());
  DLM_REQUIRE(cos_t_ && sin_t_, DLM_ERR_NOMEM, "bitnet_create: out of device memory");
  DLM_CHECK_CUDA(cudaMemcpyAsync(cos_t_, ct.data(), ct.size() * 8, cudaMemcpyHostToDevice, s));
  DLM_CHECK_CUDA(cudaMemcpyAsync(sin_t_, st.data(), st.size() * 8, cudaMemcpyHostToDevice, s));
  DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

// Activation buffers for B sequences, prefill of up to P positions, sequences of up to Lmax.
int BitNetLM::plan(int B, int P, int Lmax, bool all_logits) {
  if (B == B_ && P == P_ && Lmax == L_ && all_logits == all_logits_ && abuf_) return DLM_OK;
  release_plan();
  const BitNetCfg& c = cfg_;
  DLM_REQUIRE(B > 0 && P > 0 && P <= Lmax && Lmax <= c.max_seq, DLM_ERR_INVALID,
              "bitnet: need 0 < P <= max_len <= max_seq (P=%d, max_len=%d, max_seq=%d)", P, Lmax,
              c.max_seq);
  const size_t M = static_cast<size_t>(B) * P;
  const int D = c.d_model, F = c.ffn_dim, V = c.vocab;
  const size_t H = D / kHeadDim;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_tok = take(static_cast<size_t>(B) * Lmax * 4);
  const size_t o_h = take(M * D * 4);
  const size_t o_xq = take(M * static_cast<size_t>(F > D ? F : D));
  const size_t o_xs = take(M * 4);
  const size_t o_y = take(M * static_cast<size_t>(3 * D > 2 * F ? 3 * D : 2 * F) * 4);
  const size_t o_q = take(M * D * 4);
  const size_t o_ao = take(M * D * 4);
  const size_t kv = static_cast<size_t>(c.n_layers) * B * H * Lmax * kHeadDim * 4;
  const size_t o_k = take(kv);
  const size_t o_v = take(kv);
  const size_t rows_lm = all_logits ? M : static_cast<size_t>(B);  // forward(): every position
  const size_t ldx = (rows_lm + kLmR - 1) / kLmR * kLmR;  // the final norm's transposed rows
  const size_t o_norm = take(ldx * D * 8);
  const size_t o_logits = take(rows_lm * V * 4);
  const size_t o_state = take(64);
  const size_t o_done = take(static_cast<size_t>(B) * 4);
  const size_t o_out = take(static_cast<size_t>(B) * Lmax * 4);
  const size_t o_len = take(static_cast<size_t>(B) * 4);
  if (cudaMalloc(&abuf_, off) != cudaSuccess) {
    cudaGetLastError();
    abuf_ = nullptr;
    set_error("bitnet: cannot allocate %zu bytes of activations", off);
    return DLM_ERR_NOMEM;
  }
  char* base = static_cast<char*>(abuf_);
  tokens_ = reinterpret_cast<int*>(base + o_tok);
  h_ = reinterpret_cast<float*>(base + o_h);
  xq_ = reinterpret_cast<int8_t*>(base + o_xq);
  xs_ = reinterpret_cast<float*>(base + o_xs);
  y_ = reinterpret_cast<float*>(base + o_y);
  q_ = reinterpret_cast<float*>(base + o_q);
  ao_ = reinterpret_cast<float*>(base + o_ao);
  kc_ = reinterpret_cast<float*>(base + o_k);
  vc_ = reinterpret_cast<float*>(base + o_v);
  normT_ = reinterpret_cast<double*>(base + o_norm);
  ldx_ = static_cast<int>(ldx);
  logits_ = reinterpret_cast<float*>(base + o_logits);
  state_ = reinterpret_cast<int*>(base + o_state);  // [0] position, [1] bad-token flag
  done_ = reinterpret_cast<int*>(base + o_done);
  out_ = reinterpret_cast<int*>(base + o_out);
  out_len_ = reinterpret_cast<int*>(base + o_len);
  arena_bytes_ = off;
  B_ = B;
  P_ = P;
  L_ = Lmax;
  all_logits_ = all_logits;
  return DLM_OK;
}

// All layers for M = B * S rows (rows of sequence b at positions base + 0..S-1; base = *pos or 0).
int BitNetLM::run_layers(int S, const int* pos, cudaStream_t s) {
  const BitNetCfg& c = cfg_;
  const int M = B_ * S, D = c.d_model, F = c.ffn_dim, H = D / kHeadDim;
  const size_t kv_layer = static_cast<size_t>(B_) * H * L_ * kHeadDim;
  const int norm_blocks = (M + kNormWarps - 1) / kNormWarps;
  const size_t norm_smem = norm_smem_bytes(D);
  const size_t swi_smem = static_cast<size_t>(F) * 4;
  const size_t attn_smem = attn_smem_bytes(L_);
  int rc = DLM_OK;
  for (int l = 0; l < c.n_layers && rc == DLM_OK; ++l) {
    const Layer& Ly = layers_[l];
    float* kc = kc_ + l * kv_layer;
    float* vc = vc_ + l * kv_layer;
    DLM_CHECK_CUDA(launch_pdl(rms_norm_kernel, dim3(norm_blocks), dim3(kNormWarps * 32), norm_smem,
        s, h_, M, D, 1, 0, Ly.attn_norm, c.rms_eps, xq_, xs_, nullptr, 0));
    if (S == 1 && pos != nullptr && M < ternary_tc_min_rows()) {
      // decode: RoPE and the K / V append in the q|k|v projection's epilogue
      const RopeQkv rq{pos, cos_t_, sin_t_, q_, kc, vc, D, L_};
      rc = ternary_gemm_qkv_rope(Ly.wqkv, Ly.aqkv, xq_, xs_, M, D, rq, s, true);
      if (rc != DLM_OK) break;
    } else {
      rc = ternary_gemm_i8(Ly.wqkv, Ly.aqkv, xq_, xs_, y_, M, 3 * D, D, s, false, true);
      if (rc != DLM_OK) break;
      DLM_CHECK_CUDA(launch_pdl(rope_kv_kernel, dim3(grid1d(static_cast<size_t>(M) * H * 32, 256)),
          dim3(256), 0, s, y_, M, S, D, pos, cos_t_, sin_t_, q_, kc, vc, L_));
    }
    if (S > 1 && L_ <= kAttnSeqMax)  // prefill: one block per (sequence, head)
      // a block stages base + S positions: S when the pass starts at position 0 (no device
      // position), which leaves room for more blocks per SM than the cache length would
      DLM_CHECK_CUDA(launch_pdl(attention_seq_kernel, dim3(B_ * H), dim3(kAttnSeqWarps * 32),
          attn_seq_smem_bytes(pos ? L_ : S), s, q_, S, D, pos, kc, vc, L_, ao_));
    else
      DLM_CHECK_CUDA(launch_pdl(attention_kernel, dim3(M * H), dim3(kAttnThreads), attn_smem, s, q_,
          M, S, D, pos, kc, vc, L_, ao_));
    rc = quantize_act_i8(ao_, M, D, xq_, xs_, s);
    if (rc == DLM_OK) rc = ternary_gemm_i8(Ly.wo, Ly.ao, xq_, xs_, h_, M, D, D, s, true, true);
    if (rc != DLM_OK) break;
    DLM_CHECK_CUDA(launch_pdl(rms_norm_kernel, dim3(norm_blocks), dim3(kNormWarps * 32), norm_smem,
        s, h_, M, D, 1, 0, Ly.ffn_norm, c.rms_eps, xq_, xs_, nullptr, 0));
    rc = ternary_gemm_i8(Ly.wgu, Ly.agu, xq_, xs_, y_, M, 2 * F, D, s, false, true);
    if (rc != DLM_OK) break;
    if (M < kSwiRowsWide)
      DLM_CHECK_CUDA(launch_pdl(swiglu_quant_kernel<512>, dim3(M), dim3(512), swi_smem, s, y_, M, F,
          xq_, xs_));
    else
      DLM_CHECK_CUDA(launch_pdl(swiglu_quant_kernel<256>, dim3(M), dim3(256), swi_smem, s, y_, M, F,
          xq_, xs_));
    rc = ternary_gemm_i8(Ly.wd, Ly.ad, xq_, xs_, h_, M, D, F, s, true, true);
  }
  if (rc == DLM_OK) DLM_CHECK_CUDA(cudaGetLastError());
  return rc;
}

// final rms_norm of `rows` rows (row r reads hidden row r * stride + off) and the lm_head logits
int BitNetLM::run_head(int rows, int stride, int off, cudaStream_t s) {
  const BitNetCfg& c = cfg_;
  const int D = c.d_model;
  DLM_REQUIRE(D % kLmK == 0 && rows <= ldx_, DLM_ERR_INVALID, "bitnet: d_model %d / head rows %d", D,
              rows);
  DLM_CHECK_CUDA(launch_pdl(rms_norm_kernel, dim3((rows + kNormWarps - 1) / kNormWarps),
      dim3(kNormWarps * 32), norm_smem_bytes(D), s, h_, rows, D, stride, off, final_norm_,
      c.rms_eps, nullptr, nullptr, normT_, ldx_));
  dim3 grid((c.vocab + kLmV - 1) / kLmV, (rows + kLmR - 1) / kLmR);
  DLM_CHECK_CUDA(launch_pdl(lm_head_kernel, dim3(grid), dim3(256), 0, s, normT_, ldx_, rows, D,
      embT_, ldv_, c.vocab, logits_));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int BitNetLM::set_smem_attrs() {
  const BitNetCfg& c = cfg_;
  const size_t norm_smem = norm_smem_bytes(c.d_model);
  const size_t swi_smem = static_cast<size_t>(c.ffn_dim) * 4;
  // the largest a launch asks for: staged V at the longest staged length, or the scores alone
  const size_t attn_smem = std::max(attn_smem_bytes(std::min(c.max_seq, kVStageMax)),
                                    attn_smem_bytes(c.max_seq));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(norm_smem)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(swiglu_quant_kernel<512>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(swi_smem)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(swiglu_quant_kernel<256>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(swi_smem)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(attn_smem)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(
      attention_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(attn_seq_smem_bytes(std::min(c.max_seq, kAttnSeqMax)))));
  return DLM_OK;
}

int BitNetLM::check_bad(cudaStream_t s) {
  int bad = 0;
  DLM_CHECK_CUDA(cudaMemcpyAsync(&bad, state_ + 1, 4, cudaMemcpyDeviceToHost, s));
  DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  DLM_REQUIRE(bad == 0, DLM_ERR_INVALID, "bitnet: token id outside [0, %d)", cfg_.vocab);
  return DLM_OK;
}

int BitNetLM::forward(const int* tokens, int B, int S, float* logits, cudaStream_t s) {
  DLM_REQUIRE(tokens && logits, DLM_ERR_INVALID, "bitnet_forward: null pointer");
  int rc = plan(B, S, S, true);
  if (rc != DLM_OK) return rc;
  if ((rc = set_smem_attrs()) != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaMemcpyAsync(tokens_, tokens, static_cast<size_t>(B) * S * 4, cudaMemcpyDefault, s));
  DLM_CHECK_CUDA(cudaMemsetAsync(state_, 0, 8, s));
  DLM_CHECK_CUDA(launch_pdl(embed_kernel, dim3(B * S), dim3(128), 0, s, tokens_, S, S, nullptr,
      embed_, cfg_.vocab, cfg_.d_model, h_, B * S, state_ + 1));
  if ((rc = run_layers(S, nullptr, s)) != DLM_OK) return rc;
  if ((rc = run_head(B * S, 1, 0, s)) != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaMemcpyAsync(logits, logits_, static_cast<size_t>(B) * S * cfg_.vocab * 4,
                                 cudaMemcpyDefault, s));
  return check_bad(s);
}

// One decode pass: feed the token at position *pos of every sequence, update the cache, logits,
// greedy step, advance *pos.
int BitNetLM::decode_step(cudaStream_t s) {
  int* pos = state_;
  DLM_CHECK_CUDA(launch_pdl(embed_kernel, dim3(B_), dim3(128), 0, s, tokens_, L_, 1, pos, embed_,
      cfg_.vocab, cfg_.d_model, h_, B_, state_ + 1));
  int rc = run_layers(1, pos, s);
  if (rc == DLM_OK) rc = run_head(B_, 1, 0, s);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(launch_pdl(greedy_kernel, dim3(B_), dim3(256), 0, s, logits_, cfg_.vocab, pos, P_,
      tokens_, L_, done_, out_, L_ - P_, out_len_));
  DLM_CHECK_CUDA(launch_pdl(inc_int_kernel, dim3(1), dim3(1), 0, s, pos));
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

int BitNetLM::generate(const int* prompts, int B, int P, int max_len, int* out, int* out_len,
                       cudaStream_t s) {
  DLM_REQUIRE(prompts && out && out_len, DLM_ERR_INVALID, "bitnet_generate: null pointer");
  int rc = plan(B, P, max_len, false);
  if (rc != DLM_OK) return rc;
  if ((rc = set_smem_attrs()) != DLM_OK) return rc;
  const int G = max_len - P;  // greedy steps
  // prompts into the token table [B, max_len]
  DLM_CHECK_CUDA(cudaMemcpy2DAsync(tokens_, static_cast<size_t>(L_) * 4, prompts, static_cast<size_t>(P) * 4,
                                   static_cast<size_t>(P) * 4, B, cudaMemcpyDefault, s));
  DLM_CHECK_CUDA(cudaMemsetAsync(state_, 0, 8, s));
  DLM_CHECK_CUDA(cudaMemsetAsync(done_, 0, static_cast<size_t>(B) * 4, s));
  DLM_CHECK_CUDA(cudaMemsetAsync(out_len_, 0, static_cast<size_t>(B) * 4, s));
  if (G > 0) {
    // prefill: all prompt positions, logits of the last one, first greedy step
    DLM_CHECK_CUDA(launch_pdl(embed_kernel, dim3(B * P), dim3(128), 0, s, tokens_, L_, P, nullptr,
        embed_, cfg_.vocab, cfg_.d_model, h_, B * P, state_ + 1));
    if ((rc = run_layers(P, nullptr, s)) != DLM_OK) return rc;
    if ((rc = run_head(B, P, P - 1, s)) != DLM_OK) return rc;
    DLM_CHECK_CUDA(launch_pdl(set_int_kernel, dim3(1), dim3(1), 0, s, state_, P - 1));
    DLM_CHECK_CUDA(launch_pdl(greedy_kernel, dim3(B), dim3(256), 0, s, logits_, cfg_.vocab, state_,
        P, tokens_, L_, done_, out_, G, out_len_));
    DLM_CHECK_CUDA(launch_pdl(inc_int_kernel, dim3(1), dim3(1), 0, s, state_));
    DLM_CHECK_CUDA(cudaGetLastError());
    // decode passes (the last greedy step needs no pass after it), replayed as one CUDA graph
    if (G > 1) {
      if (!step_graph_) {
        if (!cap_stream_) DLM_CHECK_CUDA(cudaStreamCreateWithFlags(&cap_stream_, cudaStreamNonBlocking));
        cudaGraph_t g = nullptr;
        DLM_CHECK_CUDA(cudaStreamBeginCapture(cap_stream_, cudaStreamCaptureModeThreadLocal));
        rc = decode_step(cap_stream_);
        cudaError_t ce = cudaStreamEndCapture(cap_stream_, &g);
        if (rc != DLM_OK) {
          if (g) cudaGraphDestroy(g);
          return rc;
        }
        DLM_CHECK_CUDA(ce);
        ce = cudaGraphInstantiate(&step_graph_, g, 0);
        cudaGraphDestroy(g);
        DLM_CHECK_CUDA(ce);
      }
      for (int t = 1; t < G; ++t) DLM_CHECK_CUDA(cudaGraphLaunch(step_graph_, s));
    }
  }
  if (G > 0)
    DLM_CHECK_CUDA(cudaMemcpyAsync(out, out_, static_cast<size_t>(B) * G * 4, cudaMemcpyDefault, s));
  DLM_CHECK_CUDA(cudaMemcpyAsync(out_len, out_len_, static_cast<size_t>(B) * 4, cudaMemcpyDefault, s));
  return check_bad(s);
}

}  // namespace dlm

// ================================================================== C ABI

extern "C" {

static dlm::BitNetCfg to_cfg(const dlm_bitnet_config* c) {
  dlm::BitNetCfg k;
  k.vocab = c->vocab;
  k.d_model = c->d_model;
  k.n_layers = c->n_layers;
  k.n_heads = c->n_heads;
  k.ffn_dim = c->ffn_dim;
  k.max_seq = c->max_seq;
  k.rope_base = c->rope_base;
  k.rms_eps = c->rms_eps;
  k.per_tensor_scale = c->per_tensor_scale;
  return k;
}

int dlm_bitnet_create(const dlm_bitnet_config* cfg, int n, const char* const* names,
                      const float* const* weights, const int64_t* numels, void** handle, void* stream) {
  DLM_REQUIRE(cfg && handle && names && weights && n > 0, DLM_ERR_INVALID, "bitnet_create: null argument");
  *handle = nullptr;
  auto* m = new (std::nothrow) dlm::BitNetLM();
  DLM_REQUIRE(m != nullptr, DLM_ERR_NOMEM, "bitnet_create: out of host memory");
  int rc = m->create(to_cfg(cfg), n, names, weights, numels, static_cast<cudaStream_t>(stream));
  if (rc != DLM_OK) {
    delete m;
    return rc;
  }
  *handle = m;
  return DLM_OK;
}

int dlm_bitnet_destroy(void* handle) {
  delete static_cast<dlm::BitNetLM*>(handle);
  return DLM_OK;
}

int dlm_bitnet_forward(void* handle, const int* tokens, int B, int S, float* logits, void* stream) {
  DLM_REQUIRE(handle, DLM_ERR_INVALID, "bitnet_forward: null handle");
  return static_cast<dlm::BitNetLM*>(handle)->forward(tokens, B, S, logits, static_cast<cudaStream_t>(stream));
}

int dlm_bitnet_generate(void* handle, const int* prompts, int B, int P, int max_len, int* out,
                        int* out_len, void* stream) {
  DLM_REQUIRE(handle, DLM_ERR_INVALID, "bitnet_generate: null handle");
  return static_cast<dlm::BitNetLM*>(handle)->generate(prompts, B, P, max_len, out, out_len,
                                                       static_cast<cudaStream_t>(stream));
}

int dlm_bitnet_weight_count(const dlm_bitnet_config* cfg) {
  if (!cfg) return 0;
  return static_cast<int>(dlm::bitnet_weight_specs(to_cfg(cfg)).size());
}

int dlm_bitnet_weight_info(const dlm_bitnet_config* cfg, int index, char* name, int name_cap,
                           int64_t* shape, int* ndim) {
  DLM_REQUIRE(cfg && name && shape && ndim && name_cap > 0, DLM_ERR_INVALID,
              "bitnet_weight_info: null argument");
  const auto specs = dlm::bitnet_weight_specs(to_cfg(cfg));
  DLM_REQUIRE(index >= 0 && index < static_cast<int>(specs.size()), DLM_ERR_INVALID,
              "bitnet_weight_info: index %d out of range", index);
  const auto& sp = specs[index];
  DLM_REQUIRE(static_cast<int>(sp.name.size()) < name_cap, DLM_ERR_INVALID,
              "bitnet_weight_info: name buffer too small");
  std::memcpy(name, sp.name.c_str(), sp.name.size() + 1);
  *ndim = static_cast<int>(sp.shape.size());
  for (int i = 0; i < 4; ++i) shape[i] = i < *ndim ? sp.shape[i] : 0;
  return DLM_OK;
}

}  // extern "C"
