// Flash attention on tcgen05 for head_dim 64 (SDXL self / cross attention).
//
// Replaces launch_attention / launch_attention_fast (reference src/kernels/attention.cuh:53-73,
// attention.cu:393, attention_fast.cu:58): out = softmax(Q K^T * scale) V with an fp32 online
// softmax and P rounded to fp16 for the P.V product (as attention_fast.cu:238 does).
//
// One CTA = one (batch, head) and two 128-query tiles T0, T1 that share every K/V tile
// (320 or 352 threads, one CTA per SM, all 512 TMEM columns):
//   warps 0..3 / 4..7  softmax of T0 / T1: thread r of the warpgroup owns query row r (TMEM
//               lane r).  Per 128-key tile j: the row max of S_j (TMEM), p = 2^(s*c - m*c), the
//               fp32 row sum, and P_j as fp16 pairs into the tile's own 64 TMEM columns, from
//               where the P.V MMA takes its A operand (no shared-memory P).  As soon as all of
//               S_j is in registers the warps release S_j's columns, so S_{j+1} = Q K_{j+1}^T is
//               computed while P_j is still being made: both warpgroups' softmaxes run at the
//               same time instead of taking turns.  O accumulates in TMEM across the KV
//               tiles (P.V with accumulate); the running max m is lazy: it only moves when a
//               row max exceeds it by more than 8 in exp2 units (p <= 2^8 otherwise), and only
//               then is O rescaled in place (TMEM load, scale, store), so most tiles never touch
//               O.  The softmax is bound by instruction issue and MUFU latency with two warps
//               per scheduler, so the scale / shift, the row sum and the O rescale run as packed
//               f32x2 FMA / add and the row max as three-input max;
//   warp 8      TMA producer: Q (both tiles) once, then K_j / V_j through a 3-stage ring;
//   warp 9      TMEM owner + single-thread MMA issuer: S_j^t = Q_t K_j^T (M=128, N=128, K=64)
//               and O_j^t = P_j^t V_j (M=128, N=64, K=128, P from TMEM, V as an MN-major
//               operand); per tile, S_{j+1} is issued as soon as the softmax has released S_j,
//               before P_j's P.V.  With more than one key tile per query block warp 9 issues
//               T0's MMAs and an eleventh warp T1's, each waiting only on its own tile's
//               barriers (one issuer for both made each tile's P.V wait for the other tile's
//               softmax: 157 -> 138 us on B2 H10 4096^2).
// The softmax of step j+1 waits for P_j's P.V (it has read P^t) before storing P_{j+1}.
// TMEM columns: S^0 [0,128), S^1 [128,256), O^0 [256,320), P^0 [320,384), O^1 [384,448),
// P^1 [448,512).
//
// Q/K/V/O are addressed through 4D tensor maps {64 (d), heads, seq, batch} with arbitrary
// strides, so the same kernel reads the token-major [B*S, ld] projections of the UNet (head h at
// column h*64, no split/merge-heads copies) and the reference's [B, H, S, 64] layout.
// Keys beyond Sk (cross-attention, Sk = 77) are masked to -inf.  No multicast loads.
#include <cuda_fp16.h>

#include "attention.h"
#include "ptx.cuh"

namespace dlm {

namespace {

constexpr int kQT = 128;       // queries per tile (one softmax warpgroup)
constexpr int kQ = 2 * kQT;    // queries per CTA
constexpr int kKV = 128;       // keys per tile
constexpr int kD = 64;         // head dim
constexpr int kKVStages = 3;
// 10 warps; 11 with a second MMA issuer (kSplit)
constexpr int attn_threads(bool split) { return split ? 352 : 320; }
constexpr int kTileBytes = kQT * kD * 2;         // 16 KB (Q, K or V tile)
constexpr uint32_t kTmemCols = 512;

constexpr int kSmemQ = 0;                                   // 2 tiles
constexpr int kSmemK = kSmemQ + 2 * kTileBytes;
constexpr int kSmemV = kSmemK + kKVStages * kTileBytes;
constexpr int kSmemBar = kSmemV + kKVStages * kTileBytes;
constexpr int kAttnSmem = kSmemBar + 256 + 1024;
static_assert(kAttnSmem <= 226 * 1024, "shared memory");


// Work of one CTA: KV tiles [j0, j1) of one group (a 256-query block of one (batch, head));
// `whole` when that is every tile of the group.
struct AttnSeg {
  int group, j0, j1;
  bool whole;
};

__device__ __forceinline__ void attn_range(long long total, int ctas, int cta, long long& a,
                                           long long& b) {
  const long long q = total / ctas, r = total % ctas;
  a = cta * q + (cta < r ? cta : r);
  b = a + q + (cta < r ? 1 : 0);
}

// CTA whose stream-K range holds tile-step `it`.
__device__ __forceinline__ int attn_cta_of(long long total, int ctas, long long it) {
  const long long q = total / ctas, r = total % ctas;
  const long long big = r * (q + 1);
  return it < big ? static_cast<int>(it / (q + 1)) : static_cast<int>(r + (it - big) / q);
}

// This CTA's segments, identical in every role: one whole group per CTA, or under stream-K the
// group pieces of its contiguous range of the groups * n_t tile-steps.
template <bool kSK>
struct AttnSegIter {
  int it, it1, n_t;
  __device__ __forceinline__ void init(const AttnParams& p, int n_tiles, int groups) {
    n_t = n_tiles;
    if (kSK) {
      long long a, b;
      attn_range(static_cast<long long>(groups) * n_t, p.sk_ctas, blockIdx.x, a, b);
      it = static_cast<int>(a);
      it1 = static_cast<int>(b);
    } else {
      it = static_cast<int>(blockIdx.x) * n_t;
      it1 = it + n_t;
    }
  }
  __device__ __forceinline__ bool next(AttnSeg& sg) {
    if (it >= it1) return false;
    if (!kSK) {
      sg.group = static_cast<int>(blockIdx.x);
      sg.j0 = 0;
      sg.j1 = n_t;
      sg.whole = true;
      it = it1;
      return true;
    }
    sg.group = it / n_t;
    sg.j0 = it - sg.group * n_t;
    const int end = it1 - it + sg.j0;
    sg.j1 = end < n_t ? end : n_t;
    sg.whole = sg.j0 == 0 && sg.j1 == n_t;
    it += sg.j1 - sg.j0;
    return true;
  }
};

// 10 or 11 warps: one SM sub-partition holds three of them, so its 16K-register slice caps the
// kernel at 168 registers per thread.  kSK: stream-K schedule (a CTA's range of tile-steps may
// cut groups, merged through the workspace); otherwise one whole group per CTA.  kSplit: one
// MMA issuer per query tile (warp 9: T0, warp 10: T1) instead of one for both; worth its extra
// warp only when a segment has more than one key tile.
template <bool kSK, bool kSplit>
__global__ void __launch_bounds__(attn_threads(kSplit), 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + kSmemQ;
  uint8_t* sK = smem + kSmemK;
  uint8_t* sV = smem + kSmemV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* q_full = bars;                    // Q of both tiles
  uint64_t* k_full = bars + 1;                // [stages]
  uint64_t* v_full = k_full + kKVStages;      // [stages]
  uint64_t* kv_empty = v_full + kKVStages;    // [stages]
  uint64_t* s_full = kv_empty + kKVStages;    // [tile]      S_j^t ready
  uint64_t* p_full = s_full + 2;              // [tile]      P_j^t stored
  uint64_t* o_full = p_full + 2;              // [tile]      P_j^t . V_j accumulated into O^t
  uint64_t* o_empty = o_full + 2;             // [tile]      O^t of a segment read out
  uint64_t* s_free = o_empty + 2;             // [tile]      S_j^t read into registers
  uint64_t* q_empty = s_free + 2;             // the last S MMAs of a segment read Q
  uint64_t* ep_bar = q_empty + 1;             // the eight softmax warps meet (stream-K merge)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ep_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q_blocks = (p.Sq + kQ - 1) / kQ;
  const int n_tiles = (p.Sk + kKV - 1) / kKV;
  const int groups = p.B * p.H * q_blocks;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, kSplit ? 2 : 1);  // one commit per MMA issuer
    mbar_init(ep_bar, 8);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 2);  // released by P.V of both tiles
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], kQT);
      mbar_init(&o_full[t], 1);
      mbar_init(&o_empty[t], kQT);
      mbar_init(&s_free[t], kQT);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  griddep_wait();  // q / k / v are written by the previous kernel

  auto decode = [&](int group, int& b, int& h, int& q0) {
    const int qb = group % q_blocks;
    const int bh = group / q_blocks;
    h = bh % p.H;
    b = bh / p.H;
    q0 = qb * kQ;
  };

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int stage = 0;
      uint32_t phase = 0;
      int seg = 0;
      bool ok = true;
      AttnSegIter<kSK> si;
      si.init(p, n_tiles, groups);
      AttnSeg sg;
      while (ok && si.next(sg)) {
        int b, h, q0;
        decode(sg.group, b, h, q0);
        // the previous segment's last S MMAs must have read Q before it is replaced
        if (seg > 0 && !mbar_wait(q_empty, (seg - 1) & 1, abort_flag, p.status, kDevTimeoutProducer))
          break;
        mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
        tma_load_4d(sQ, &tmQ, q_full, 0, h, q0, b);
        tma_load_4d(sQ + kTileBytes, &tmQ, q_full, 0, h, q0 + kQT, b);
        for (int j = sg.j0; j < sg.j1; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[stage], kTileBytes);
          tma_load_4d(sK + stage * kTileBytes, &tmK, &k_full[stage], 0, h, j * kKV, b);
          mbar_arrive_expect_tx(&v_full[stage], kTileBytes);
          tma_load_4d(sV + stage * kTileBytes, &tmV, &v_full[stage], 0, h, j * kKV, b);
          if (++stage == kKVStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        ++seg;
      }
    }
  } else if (warp == 9 || (kSplit && warp == 10)) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kQT, kKV, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(kQT, kD, true);
      int kc = 0;   // KV tiles consumed so far (ring stage / phase)
      int jc = 0;   // tile-steps so far (S / P / O phases)
      int seg = 0;
      bool ok = true;
      auto issue_s = [&](int t, int jl) -> bool {
        const int kk = kc + jl, st = kk % kKVStages;
        const int step = jc + jl;
        // S^t is free once the softmax warps hold the previous tile-step's S in registers
        if (step > 0 &&
            !mbar_wait(&s_free[t], (step - 1) & 1, abort_flag, p.status, kDevTimeoutMma))
          return false;
        if (!mbar_wait(&k_full[st], (kk / kKVStages) & 1, abort_flag, p.status, kDevTimeoutMma))
          return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + t * kTileBytes);
        const uint32_t k_addr = smem_u32(sK + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          umma_f16_ss(tbase + t * kKV, sw128_desc(q_addr + k * 32, 16, 1024),
                      sw128_desc(k_addr + k * 32, 16, 1024), idesc_s, k != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
        return true;
      };
      auto issue_pv = [&](int t, int jl) -> bool {
        const int kk = kc + jl, st = kk % kKVStages;
        if (!mbar_wait(&v_full[st], (kk / kKVStages) & 1, abort_flag, p.status, kDevTimeoutMma))
          return false;
        // O^t accumulates over the segment; its first P.V overwrites it once the softmax warps
        // have read out the previous segment's O
        if (jl == 0 && seg > 0 &&
            !mbar_wait(&o_empty[t], (seg - 1) & 1, abort_flag, p.status, kDevTimeoutMma))
          return false;
        tc_fence_after();
        const uint32_t p_tmem = tbase + 320 + t * 128;  // P^t: 64 columns of fp16 pairs
        const uint32_t v_addr = smem_u32(sV + st * kTileBytes);
        const uint32_t d = tbase + 256 + t * 128;
#pragma unroll
        for (int ks = 0; ks < kKV / 16; ++ks) {
          const uint64_t bd = sw128_desc(v_addr + ks * 2048, 1024, 1024);
          umma_f16_ts(d, p_tmem + ks * 8, bd, idesc_o, (jl != 0 || ks != 0) ? 1u : 0u);
        }
        umma_commit(&o_full[t]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      if constexpr (kSplit) {
        // One issuing thread per query tile (warp 9: T0, warp 10: T1), so neither tile's MMAs
        // wait behind the other tile's softmax: S_{j+1} once S_j is released, then P_j.V once
        // P_j is stored.  The two issuers share the K / V ring (each commits kv_empty once per
        // stage) and Q (each commits q_empty once per segment).
        const int t = warp - 9;
        AttnSegIter<kSK> si;
        si.init(p, n_tiles, groups);
        AttnSeg sg;
        while (ok && si.next(sg)) {
          const int n = sg.j1 - sg.j0;
          ok = mbar_wait(q_full, seg & 1, abort_flag, p.status, kDevTimeoutMma);
          if (ok) ok = issue_s(t, 0);
          if (ok && n == 1) umma_commit(q_empty);  // Q is not read after this
          for (int jl = 0; jl < n && ok; ++jl) {
            if (jl + 1 < n) {
              ok = issue_s(t, jl + 1);
              if (ok && jl + 2 == n) umma_commit(q_empty);  // last S of the segment
            }
            if (ok && !mbar_wait(&p_full[t], (jc + jl) & 1, abort_flag, p.status, kDevTimeoutMma))
              ok = false;
            if (!ok) break;
            tc_fence_after();
            ok = issue_pv(t, jl);
          }
          kc += n;
          jc += n;
          ++seg;
        }
      } else {
        // one issuer for both tiles, per key tile: each tile's S_{j+1} (once S_j is released),
        // then its P_j.V (once P_j is stored)
        AttnSegIter<kSK> si;
        si.init(p, n_tiles, groups);
        AttnSeg sg;
        while (ok && si.next(sg)) {
          const int n = sg.j1 - sg.j0;
          ok = mbar_wait(q_full, seg & 1, abort_flag, p.status, kDevTimeoutMma);
          if (ok) ok = issue_s(0, 0);
          if (ok) ok = issue_s(1, 0);
          if (ok && n == 1) umma_commit(q_empty);  // Q is not read after these
          for (int jl = 0; jl < n && ok; ++jl) {
            for (int t = 0; t < 2 && ok; ++t) {
              if (jl + 1 < n) {
                ok = issue_s(t, jl + 1);
                if (ok && t == 1 && jl + 2 == n) umma_commit(q_empty);  // last S of the segment
              }
              if (ok &&
                  !mbar_wait(&p_full[t], (jc + jl) & 1, abort_flag, p.status, kDevTimeoutMma))
                ok = false;
              if (!ok) break;
              tc_fence_after();
              ok = issue_pv(t, jl);
            }
          }
          kc += n;
          jc += n;
          ++seg;
        }
      }
      // the last MMA is issued: the next kernel may launch during this CTA's final softmax
      griddep_launch_dependents();
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..7
    const int t = warp >> 2;                       // query tile of this warpgroup
    const int row = (warp & 3) * 32 + lane;        // TMEM lane == query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t ts = tbase + lane_off + t * kKV;
    const uint32_t to = tbase + lane_off + 256 + t * 128;
    const uint32_t tp = tbase + lane_off + 320 + t * 128;
    // S_j^t is in this thread's registers: the MMA warp may write S_{j+1}^t
    auto release_s = [&]() {
      tc_fence_before();
      mbar_arrive(&s_free[t]);
    };
    const float c = p.scale_log2;
    bool ok = true;
    int jc = 0;
    uint32_t ep_phase = 0;
    // the eight softmax warps meet (bounded)
    auto ep_meet = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(ep_bar);
      const bool r = mbar_wait(ep_bar, ep_phase, abort_flag, p.status, kDevTimeoutSoftmax);
      ep_phase ^= 1;
      return r;
    };

    // bounded wait whose outcome is the same in every lane (the warp-collective TMEM accesses
    // that follow need all 32 lanes)
    auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, kDevTimeoutSoftmax));
    };
    // O^t *= alpha in place (this warp's 32 rows), for rows whose running max moved
    auto rescale_o = [&](float alpha) {
      uint32_t r0[32], r1[32];
      tmem_ld_32x32b_x32(to, r0);
      tmem_ld_32x32b_x32(to + 32, r1);
      tmem_ld_wait();
      const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
      for (int q = 0; q < 32; q += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r0[q]), __uint_as_float(r0[q + 1])), a2, f2_pack(0.0f, 0.0f)), x0, x1);
        r0[q] = __float_as_uint(x0);
        r0[q + 1] = __float_as_uint(x1);
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r1[q]), __uint_as_float(r1[q + 1])), a2, f2_pack(0.0f, 0.0f)), x0, x1);
        r1[q] = __float_as_uint(x0);
        r1[q + 1] = __float_as_uint(x1);
      }
      tmem_st_32x32b_x32(to, r0);
      tmem_st_32x32b_x32(to + 32, r1);
      tmem_st_wait();
    };

    AttnSegIter<kSK> si;
    si.init(p, n_tiles, groups);
    AttnSeg sg;
    while (ok && si.next(sg)) {
      const int n = sg.j1 - sg.j0;
      float m_run = -INFINITY, l_run = 0.0f;

      for (int jl = 0; jl < n; ++jl) {
        const int jj = jc + jl;
        if (!wwait(&s_full[t], jj & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int valid = p.Sk - (sg.j0 + jl) * kKV;  // keys of this tile (may exceed 128)
        const bool full_tile = valid >= kKV;
        if (jl >= 1 && full_tile) {
          // One pass over S, 32 columns at a time, each chunk's TMEM load issued while the
          // previous chunk is exponentiated (so its latency hides behind that work): the chunk's
          // row max is checked against the running max m (the same lazy rule: m moves only when
          // the max exceeds it by more than 8 in exp2 units, so p = 2^(s c - m c) <= 2^8), then
          // exponentiated against m and its fp16 P stored.  A move at chunk k rescales the partial
          // sums at once and, after the pass, the P of the chunks before k already in TMEM, and
          // (after the previous P.V) O.
          float m_cur = m_run, alpha_all = 1.0f;
          float a_after[3] = {1.0f, 1.0f, 1.0f};  // scale still owed by the P of chunk 0, 1, 2
          uint64_t sumA = f2_pack(0.0f, 0.0f), sumB = sumA;
          uint32_t buf[2][32];
          bool waited = true;
          tmem_ld_32x32b_x32(ts, buf[0]);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (k < 3) tmem_ld_32x32b_x32(ts + (k + 1) * 32, buf[(k + 1) & 1]);  // prefetch
            const uint32_t* r = buf[k & 1];
            float h0 = m_cur, h1 = m_cur;
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              h0 = max3f(h0, __uint_as_float(r[q]), __uint_as_float(r[q + 1]));
              h1 = max3f(h1, __uint_as_float(r[q + 2]), __uint_as_float(r[q + 3]));
            }
            const float hm = fmaxf(h0, h1);
            if ((hm - m_cur) * c > 8.0f) {
              const float a = fast_exp2((m_cur - hm) * c);
              alpha_all *= a;
#pragma unroll
              for (int j = 0; j < 3; ++j)
                if (j < k) a_after[j] *= a;
              const uint64_t a2 = f2_pack(a, a), z2 = f2_pack(0.0f, 0.0f);
              sumA = f2_fma(sumA, a2, z2);
              sumB = f2_fma(sumB, a2, z2);
              m_cur = hm;
            }
            const float mcc = m_cur * c;
            const uint64_t c2 = f2_pack(c, c), nmc2 = f2_pack(-mcc, -mcc);
            uint32_t pp[16];
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(r[q]), __uint_as_float(r[q + 1])), c2, nmc2),
                        x0, x1);
              const float e0 = fast_exp2(x0);
              const float e1 = fast_exp2(x1);
              if (q & 2)
                sumB = f2_add(sumB, f2_pack(e0, e1));
              else
                sumA = f2_add(sumA, f2_pack(e0, e1));
              pp[q >> 1] = pack_half2(e0, e1);
            }
            if (k == 0) {
              // P_{j-1}.V is complete: it has read P^t and added into O
              waited = wwait(&o_full[t], (jj - 1) & 1);
              if (!waited) {
                tmem_ld_wait();
                break;
              }
              tc_fence_after();
            }
            tmem_st_32x32b_x16(tp + k * 16, pp);
            if (k < 3) tmem_ld_wait();  // the prefetched chunk has arrived
            if (k == 2) release_s();    // all of S_j is in registers
          }
          if (!waited) {
            ok = false;
            break;
          }
          tmem_st_wait();
#pragma unroll
          for (int k = 0; k < 3; ++k) {
            if (__any_sync(0xffffffffu, a_after[k] != 1.0f)) {
              // chunk k's P was written against a max that a later chunk moved
              uint32_t pp[16];
              tmem_ld_32x32b_x16(tp + k * 16, pp);
              tmem_ld_wait();
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pp[q]));
                pp[q] = pack_half2(f.x * a_after[k], f.y * a_after[k]);
              }
              tmem_st_32x32b_x16(tp + k * 16, pp);
              tmem_st_wait();
            }
          }
          if (__any_sync(0xffffffffu, alpha_all != 1.0f)) rescale_o(alpha_all);
          float sum0, sum1, sum2, sum3;
          f2_unpack(sumA, sum0, sum1);
          f2_unpack(sumB, sum2, sum3);
          tc_fence_before();
          mbar_arrive(&p_full[t]);
          l_run = fmaf(l_run, alpha_all, (sum0 + sum1) + (sum2 + sum3));
          m_run = m_cur;
          continue;
        }
        // pass 1: row max over 128 columns, two TMEM loads in flight, four independent chains
        float mx0 = m_run, mx1 = m_run, mx2 = m_run, mx3 = m_run;
#pragma unroll
        for (int cc = 0; cc < 4; cc += 2) {
          uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(ts + cc * 32, ra);
          tmem_ld_32x32b_x32(ts + cc * 32 + 32, rb);
          tmem_ld_wait();
          if (full_tile) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              mx0 = max3f(mx0, __uint_as_float(ra[q]), __uint_as_float(ra[q + 1]));
              mx1 = max3f(mx1, __uint_as_float(ra[q + 2]), __uint_as_float(ra[q + 3]));
              mx2 = max3f(mx2, __uint_as_float(rb[q]), __uint_as_float(rb[q + 1]));
              mx3 = max3f(mx3, __uint_as_float(rb[q + 2]), __uint_as_float(rb[q + 3]));
            }
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              if (cc * 32 + q < valid) mx0 = fmaxf(mx0, __uint_as_float(ra[q]));
              if (cc * 32 + 32 + q < valid) mx1 = fmaxf(mx1, __uint_as_float(rb[q]));
            }
          }
        }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        // Lazy rescale: the running max m_run only moves when a row's max exceeds it by more
        // than 8 in exp2 units (so p = 2^(s c - m c) <= 2^8 stays exact in fp16 range); then O
        // and the row sum are scaled by alpha = 2^((m_old - m_new) c).
        float m_new = m_run, alpha = 1.0f;
        if (jl == 0) {
          m_new = mx;
        } else if ((mx - m_run) * c > 8.0f) {
          m_new = mx;
          alpha = fast_exp2((m_run - mx) * c);
        }
        const float mc = m_new * c;
        if (jl >= 1) {
          // P.V of tile j-1 is complete: it has read the P buffer and added into O
          if (!wwait(&o_full[t], (jj - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, alpha != 1.0f)) rescale_o(alpha);
        }
        // pass 2: p = exp2(s*c - m*c), fp32 row sum, fp16 P (pairs of consecutive keys) into P^t
        const uint64_t c2 = f2_pack(c, c), nmc2 = f2_pack(-mc, -mc);
        uint64_t sumA = f2_pack(0.0f, 0.0f), sumB = sumA;
#pragma unroll
        for (int cc = 0; cc < 4; cc += 2) {
          uint32_t ra[32], rb[32];
          tmem_ld_32x32b_x32(ts + cc * 32, ra);
          tmem_ld_32x32b_x32(ts + cc * 32 + 32, rb);
          tmem_ld_wait();
          if (cc == 2) release_s();
          uint32_t pp[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint32_t* r = half ? rb : ra;
            const int col0 = (cc + half) * 32;
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(r[q]), __uint_as_float(r[q + 1])), c2, nmc2),
                        x0, x1);
              float e0 = fast_exp2(x0);
              float e1 = fast_exp2(x1);
              if (!full_tile) {
                if (col0 + q >= valid) e0 = 0.0f;
                if (col0 + q + 1 >= valid) e1 = 0.0f;
              }
              if (q & 2)
                sumB = f2_add(sumB, f2_pack(e0, e1));
              else
                sumA = f2_add(sumA, f2_pack(e0, e1));
              pp[half * 16 + (q >> 1)] = pack_half2(e0, e1);
            }
          }
          tmem_st_32x32b_x32(tp + (cc >> 1) * 32, pp);
        }
        tmem_st_wait();
        float sum0, sum1, sum2, sum3;
        f2_unpack(sumA, sum0, sum1);
        f2_unpack(sumB, sum2, sum3);
        tc_fence_before();
        mbar_arrive(&p_full[t]);
        l_run = fmaf(l_run, alpha, (sum0 + sum1) + (sum2 + sum3));
        m_run = m_new;
      }
      if (ok && n > 0) ok = wwait(&o_full[t], (jc + n - 1) & 1);  // the segment's last P.V
      jc += n;
      if (!ok) break;
      if (n == 0) continue;
      tc_fence_after();
      int b, h, q0;
      decode(sg.group, b, h, q0);
      const int qrow = q0 + t * kQT + row;
      __half* dst = p.out + static_cast<size_t>(b) * p.o_sb + static_cast<size_t>(h) * p.o_sh +
                    static_cast<size_t>(qrow) * p.o_ss;
      // a group cut between CTAs (stream-K): this piece goes to the workspace, normalised by its
      // own row sum, and the last CTA to finish merges the pieces
      // a cut query block (stream-K); with one key tile per block (not kSplit) none is ever cut
      const bool piece = kSK && kSplit && !sg.whole;
      const int r_in = t * kQT + row;
      int first = 0, last = 0;
      if (piece) {
        const long long total = static_cast<long long>(groups) * n_tiles;
        first = attn_cta_of(total, p.sk_ctas, static_cast<long long>(sg.group) * n_tiles);
        last = attn_cta_of(total, p.sk_ctas, static_cast<long long>(sg.group + 1) * n_tiles - 1);
      }
      auto slot_of = [&](int cc) { return 2 * cc + (cc == first ? 1 : 0); };
      const size_t my_slot = static_cast<size_t>(slot_of(static_cast<int>(blockIdx.x))) * kQ + r_in;
      if (piece && sg.j0 == 0) {
        // The last piece of a cut query block, when every other piece is already in the workspace
        // (their CTAs have counted them): merge straight from this CTA's O in TMEM, without
        // writing and re-reading its own piece.  This CTA does not count itself, so no other can
        // also find itself last; otherwise the counted path below runs as before.  Only a block's
        // head piece checks: it ends its CTA's range, while the tail pieces, which begin theirs,
        // finish early and are almost never last.
        ok = ep_meet();
        if (!ok) break;
        if (threadIdx.x == 0) {
          int cnt;
          asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(cnt) : "l"(p.part_cnt + sg.group) : "memory");
          *last_flag = cnt == last - first;
        }
        ok = ep_meet();
        if (!ok) break;
        if (*last_flag) {
          const int me = static_cast<int>(blockIdx.x);
          float mmax = m_run;
          for (int cc = first; cc <= last; ++cc)
            if (cc != me) mmax = fmaxf(mmax, __ldcg(p.part_ml + static_cast<size_t>(slot_of(cc)) * kQ + r_in).x);
          // own O is unnormalised (sum of 2^((s - m) c) v): its weight l 2^((m - M) c) over l
          const float so = fast_exp2((m_run - mmax) * c);
          float L = l_run * so;
          for (int cc = first; cc <= last; ++cc) {
            if (cc == me) continue;
            const float2 ml = __ldcg(p.part_ml + static_cast<size_t>(slot_of(cc)) * kQ + r_in);
            L += ml.y * fast_exp2((ml.x - mmax) * c);
          }
          const float inv = 1.0f / L;
#pragma unroll 1
          for (int qd = 0; qd < 4; ++qd) {  // 16 columns at a time
            uint32_t r[16];
            tmem_ld_32x32b_x16(to + qd * 16, r);
            tmem_ld_wait();
            float a16[16];
#pragma unroll
            for (int d = 0; d < 16; ++d) a16[d] = __uint_as_float(r[d]) * so;
            for (int cc = first; cc <= last; ++cc) {
              if (cc == me) continue;
              const size_t sl = static_cast<size_t>(slot_of(cc)) * kQ + r_in;
              const float2 ml = __ldcg(p.part_ml + sl);
              const uint4* po = reinterpret_cast<const uint4*>(p.part_o + sl * kD) + 2 * qd;
              const uint4 o0 = __ldcg(po), o1 = __ldcg(po + 1);
              const float w = ml.y * fast_exp2((ml.x - mmax) * c);
              const __half2* h0 = reinterpret_cast<const __half2*>(&o0);
              const __half2* h1 = reinterpret_cast<const __half2*>(&o1);
#pragma unroll
              for (int k2 = 0; k2 < 4; ++k2) {
                const float2 f0 = __half22float2(h0[k2]), f1 = __half22float2(h1[k2]);
                a16[2 * k2] = fmaf(w, f0.x, a16[2 * k2]);
                a16[2 * k2 + 1] = fmaf(w, f0.y, a16[2 * k2 + 1]);
                a16[8 + 2 * k2] = fmaf(w, f1.x, a16[8 + 2 * k2]);
                a16[8 + 2 * k2 + 1] = fmaf(w, f1.y, a16[8 + 2 * k2 + 1]);
              }
            }
            if (qrow < p.Sq) {
              uint4 v0, v1;
              v0.x = pack_half2(a16[0] * inv, a16[1] * inv);
              v0.y = pack_half2(a16[2] * inv, a16[3] * inv);
              v0.z = pack_half2(a16[4] * inv, a16[5] * inv);
              v0.w = pack_half2(a16[6] * inv, a16[7] * inv);
              v1.x = pack_half2(a16[8] * inv, a16[9] * inv);
              v1.y = pack_half2(a16[10] * inv, a16[11] * inv);
              v1.z = pack_half2(a16[12] * inv, a16[13] * inv);
              v1.w = pack_half2(a16[14] * inv, a16[15] * inv);
              *reinterpret_cast<uint4*>(dst + 16 * qd) = v0;
              *reinterpret_cast<uint4*>(dst + 16 * qd + 8) = v1;
            }
          }
          tc_fence_before();
          mbar_arrive(&o_empty[t]);
          if (threadIdx.x == 0) p.part_cnt[sg.group] = 0;
          continue;
        }
      }
      {
        // O leaves TMEM 32 columns at a time (fp16, scaled by 1 / l), then the next segment's
        // first P.V may overwrite it
        const float inv = 1.0f / l_run;
        uint4* po = reinterpret_cast<uint4*>(p.part_o + my_slot * kD);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(to + hf * 32, r);
          tmem_ld_wait();
          uint4 v[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[j].x = pack_half2(__uint_as_float(r[8 * j]) * inv, __uint_as_float(r[8 * j + 1]) * inv);
            v[j].y = pack_half2(__uint_as_float(r[8 * j + 2]) * inv, __uint_as_float(r[8 * j + 3]) * inv);
            v[j].z = pack_half2(__uint_as_float(r[8 * j + 4]) * inv, __uint_as_float(r[8 * j + 5]) * inv);
            v[j].w = pack_half2(__uint_as_float(r[8 * j + 6]) * inv, __uint_as_float(r[8 * j + 7]) * inv);
          }
          if (piece) {
#pragma unroll
            for (int j = 0; j < 4; ++j) __stcg(po + 4 * hf + j, v[j]);
          } else if (qrow < p.Sq) {
#pragma unroll
            for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(dst + 32 * hf + 8 * j) = v[j];
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty[t]);
      }
      if (!piece) continue;
      __stcg(p.part_ml + my_slot, make_float2(m_run, l_run));
      __threadfence();
      ok = ep_meet();
      if (!ok) break;
      if (threadIdx.x == 0) {
        const int old = atomicAdd(p.part_cnt + sg.group, 1);
        *last_flag = old == last - first;
      }
      ok = ep_meet();
      if (!ok) break;
      if (*last_flag) {
        __threadfence();
        // merge the pieces in CTA order: O = sum_s w_s O_s / sum_s w_s, w_s = l_s 2^((m_s - m) c),
        // 32 columns at a time; the (max, sum) pairs of up to four pieces are requested before
        // any is used
        float mmax = -INFINITY;
        for (int c0 = first; c0 <= last; c0 += 4) {
          float2 m4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (c0 + i <= last) m4[i] = __ldcg(p.part_ml + static_cast<size_t>(slot_of(c0 + i)) * kQ + r_in);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (c0 + i <= last) mmax = fmaxf(mmax, m4[i].x);
        }
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          float a32[32];
#pragma unroll
          for (int d = 0; d < 32; ++d) a32[d] = 0.0f;
          float L = 0.0f;
          for (int cc = first; cc <= last; ++cc) {
            const size_t sl = static_cast<size_t>(slot_of(cc)) * kQ + r_in;
            const float2 ml = __ldcg(p.part_ml + sl);
            const uint4* po = reinterpret_cast<const uint4*>(p.part_o + sl * kD) + 4 * hf;
            uint4 ov[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) ov[j] = __ldcg(po + j);
            const float w = ml.y * fast_exp2((ml.x - mmax) * c);
            L += w;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __half2* hh = reinterpret_cast<const __half2*>(&ov[j]);
#pragma unroll
              for (int k2 = 0; k2 < 4; ++k2) {
                const float2 f = __half22float2(hh[k2]);
                a32[8 * j + 2 * k2] = fmaf(w, f.x, a32[8 * j + 2 * k2]);
                a32[8 * j + 2 * k2 + 1] = fmaf(w, f.y, a32[8 * j + 2 * k2 + 1]);
              }
            }
          }
          if (qrow < p.Sq) {
            const float inv = 1.0f / L;
#pragma unroll
            for (int d = 0; d < 32; d += 8) {
              uint4 v;
              v.x = pack_half2(a32[d] * inv, a32[d + 1] * inv);
              v.y = pack_half2(a32[d + 2] * inv, a32[d + 3] * inv);
              v.z = pack_half2(a32[d + 4] * inv, a32[d + 5] * inv);
              v.w = pack_half2(a32[d + 6] * inv, a32[d + 7] * inv);
              *reinterpret_cast<uint4*>(dst + 32 * hf + d) = v;
            }
          }
        }
        if (threadIdx.x == 0) p.part_cnt[sg.group] = 0;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

bool make_qkv_map(CUtensorMap* m, const __half* base, const AttnTensor& t, int B, int H, int S) {
  const uint64_t dims[4] = {64, static_cast<uint64_t>(H), static_cast<uint64_t>(S),
                            static_cast<uint64_t>(B)};
  const uint64_t st[3] = {static_cast<uint64_t>(t.sh) * 2, static_cast<uint64_t>(t.ss) * 2,
                          static_cast<uint64_t>(t.sb) * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims, st, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

bool stride_ok(const AttnTensor& t) {
  return (reinterpret_cast<uintptr_t>(t.ptr) & 15) == 0 && t.sh % 8 == 0 && t.ss % 8 == 0 &&
         t.sb % 8 == 0 && t.sh > 0 && t.ss > 0 && t.sb > 0;
}

}  // namespace

size_t attn_counter_bytes(int B, int H, int Sq) {
  const size_t groups = static_cast<size_t>(B) * H * ((Sq + kQ - 1) / kQ);
  return ((groups * sizeof(int) + 255) / 256) * 256;
}

size_t attn_workspace_bytes(int B, int H, int Sq) {
  const size_t slots = 2 * static_cast<size_t>(num_sms());
  return attn_counter_bytes(B, H, Sq) + slots * kQ * sizeof(float2) + slots * kQ * kD * sizeof(__half);
}

int attn_plan(AttnOp* op, int B, int H, int Sq, int Sk, int Dh, float scale, const AttnTensor& q,
              const AttnTensor& k, const AttnTensor& v, const AttnTensor& o, void* ws,
              size_t ws_bytes) {
  DLM_REQUIRE(op != nullptr, DLM_ERR_INVALID, "attention: null op");
  DLM_REQUIRE(B > 0 && H > 0 && Sq > 0 && Sk > 0, DLM_ERR_INVALID, "attention: empty problem");
  DLM_REQUIRE(Dh == 64, DLM_ERR_UNSUPPORTED, "attention: head_dim %d (only 64 here)", Dh);
  DLM_REQUIRE(q.ptr && k.ptr && v.ptr && o.ptr, DLM_ERR_INVALID, "attention: null tensor");
  DLM_REQUIRE(stride_ok(q) && stride_ok(k) && stride_ok(v) && stride_ok(o), DLM_ERR_INVALID,
              "attention: tensors must be 16-byte aligned with strides %% 8 == 0");
  std::memset(op, 0, sizeof(*op));
  if (!make_qkv_map(&op->tmQ, q.ptr, q, B, H, Sq)) return DLM_ERR_CUDA;
  if (!make_qkv_map(&op->tmK, k.ptr, k, B, H, Sk)) return DLM_ERR_CUDA;
  if (!make_qkv_map(&op->tmV, v.ptr, v, B, H, Sk)) return DLM_ERR_CUDA;
  AttnParams& p = op->p;
  p.B = B;
  p.H = H;
  p.Sq = Sq;
  p.Sk = Sk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = const_cast<__half*>(o.ptr);
  p.o_sb = o.sb;
  p.o_sh = o.sh;
  p.o_ss = o.ss;
  p.status = device_status_ptr();
  const long long groups = static_cast<long long>(B) * H * ((Sq + kQ - 1) / kQ);
  const long long steps = groups * ((Sk + kKV - 1) / kKV);
  DLM_REQUIRE(steps < (1ll << 31), DLM_ERR_INVALID, "attention: too many query blocks x key tiles");
  op->grid = static_cast<int>(groups);
  if (ws != nullptr) {
    // stream-K: every SM takes an equal share of the groups' KV tile-steps
    DLM_REQUIRE((reinterpret_cast<uintptr_t>(ws) & 255) == 0, DLM_ERR_INVALID,
                "attention: workspace must be 256-byte aligned");
    DLM_REQUIRE(ws_bytes >= attn_workspace_bytes(B, H, Sq), DLM_ERR_INVALID,
                "attention: workspace of %zu bytes, need %zu", ws_bytes, attn_workspace_bytes(B, H, Sq));
    const int sms = num_sms();
    p.sk_ctas = static_cast<int>(steps < sms ? steps : sms);
    char* base = static_cast<char*>(ws);
    p.part_cnt = reinterpret_cast<int*>(base);
    base += attn_counter_bytes(B, H, Sq);
    p.part_ml = reinterpret_cast<float2*>(base);
    base += 2 * static_cast<size_t>(sms) * kQ * sizeof(float2);
    p.part_o = reinterpret_cast<__half*>(base);
    op->grid = p.sk_ctas;
  }
  return DLM_OK;
}

int attn_prepare_kernels() {
  const void* fns[4] = {reinterpret_cast<const void*>(attn_fwd_kernel<false, false>),
                        reinterpret_cast<const void*>(attn_fwd_kernel<true, false>),
                        reinterpret_cast<const void*>(attn_fwd_kernel<false, true>),
                        reinterpret_cast<const void*>(attn_fwd_kernel<true, true>)};
  for (const void* f : fns)
    DLM_CHECK_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
  return DLM_OK;
}

int attn_launch(const AttnOp& op, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const int rc = attn_prepare_kernels();
    if (rc != DLM_OK) return rc;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  const bool split = op.p.Sk > kKV;  // more than one key tile per query block
  cfg.blockDim = dim3(attn_threads(split), 1, 1);
  cfg.dynamicSmemBytes = kAttnSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const bool sk = op.p.sk_ctas > 0;
  if (sk && split)
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_fwd_kernel<true, true>, op.tmQ, op.tmK, op.tmV, op.p));
  else if (sk)
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_fwd_kernel<true, false>, op.tmQ, op.tmK, op.tmV, op.p));
  else if (split)
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_fwd_kernel<false, true>, op.tmQ, op.tmK, op.tmV, op.p));
  else
    DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_fwd_kernel<false, false>, op.tmQ, op.tmK, op.tmV, op.p));
  return DLM_OK;
}

}  // namespace dlm

extern "C" {

int dlm_launch_attention(const void* q, const void* k, const void* v, void* out, int B, int H,
                         int Sq, int Sk, int Dh, float scale, void* stream) {
  if (B == 0 || H == 0 || Sq == 0 || Sk == 0) return DLM_OK;
  // reference layout [B, H, S, Dh] contiguous (src/kernels/attention.cuh:11-20)
  auto bhsd = [&](const void* ptr, int S) {
    dlm::AttnTensor t;
    t.ptr = static_cast<const __half*>(ptr);
    t.ss = Dh;
    t.sh = static_cast<long long>(S) * Dh;
    t.sb = static_cast<long long>(H) * S * Dh;
    return t;
  };
  if (Dh != 64) {  // wide heads (the VAE's Dh = 512)
    dlm::AttnWideOp op;
    int rc = dlm::attn_wide_plan(&op, B, H, Sq, Sk, Dh, scale, bhsd(q, Sq), bhsd(k, Sk),
                                 bhsd(v, Sk), bhsd(out, Sq));
    if (rc != DLM_OK) return rc;
    return dlm::attn_wide_launch(op, static_cast<cudaStream_t>(stream));
  }
  dlm::AttnOp op;
  int rc = dlm::attn_plan(&op, B, H, Sq, Sk, Dh, scale, bhsd(q, Sq), bhsd(k, Sk), bhsd(v, Sk),
                          bhsd(out, Sq));
  if (rc != DLM_OK) return rc;
  return dlm::attn_launch(op, static_cast<cudaStream_t>(stream));
}

size_t dlm_attention_workspace_bytes(int B, int H, int Sq) {
  return dlm::attn_workspace_bytes(B, H, Sq);
}

int dlm_launch_attention_ws(const void* q, const void* k, const void* v, void* out, int B, int H,
                            int Sq, int Sk, int Dh, float scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (B == 0 || H == 0 || Sq == 0 || Sk == 0) return DLM_OK;
  auto bhsd = [&](const void* ptr, int S) {
    dlm::AttnTensor t;
    t.ptr = static_cast<const __half*>(ptr);
    t.ss = Dh;
    t.sh = static_cast<long long>(S) * Dh;
    t.sb = static_cast<long long>(H) * S * Dh;
    return t;
  };
  if (Dh != 64) {  // wide heads: no stream-K, the workspace is not used
    dlm::AttnWideOp op;
    int rc = dlm::attn_wide_plan(&op, B, H, Sq, Sk, Dh, scale, bhsd(q, Sq), bhsd(k, Sk),
                                 bhsd(v, Sk), bhsd(out, Sq));
    if (rc != DLM_OK) return rc;
    return dlm::attn_wide_launch(op, static_cast<cudaStream_t>(stream));
  }
  dlm::AttnOp op;
  int rc = dlm::attn_plan(&op, B, H, Sq, Sk, Dh, scale, bhsd(q, Sq), bhsd(k, Sk), bhsd(v, Sk),
                          bhsd(out, Sq), workspace, workspace_bytes);
  if (rc != DLM_OK) return rc;
  return dlm::attn_launch(op, static_cast<cudaStream_t>(stream));
}

int dlm_attention_tokens(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv,
                         void* out, int ldo, int B, int H, int Sq, int Sk, int Dh, float scale,
                         void* stream) {
  if (B == 0 || H == 0 || Sq == 0 || Sk == 0) return DLM_OK;
  auto tok = [&](const void* ptr, int ld, int S) {
    dlm::AttnTensor t;
    t.ptr = static_cast<const __half*>(ptr);
    t.ss = ld;
    t.sh = Dh;
    t.sb = static_cast<long long>(S) * ld;
    return t;
  };
  if (Dh != 64) {  // wide heads
    dlm::AttnWideOp op;
    int rc = dlm::attn_wide_plan(&op, B, H, Sq, Sk, Dh, scale, tok(q, ldq, Sq), tok(k, ldk, Sk),
                                 tok(v, ldv, Sk), tok(out, ldo, Sq));
    if (rc != DLM_OK) return rc;
    return dlm::attn_wide_launch(op, static_cast<cudaStream_t>(stream));
  }
  dlm::AttnOp op;
  int rc = dlm::attn_plan(&op, B, H, Sq, Sk, Dh, scale, tok(q, ldq, Sq), tok(k, ldk, Sk),
                          tok(v, ldv, Sk), tok(out, ldo, Sq));
  if (rc != DLM_OK) return rc;
  return dlm::attn_launch(op, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
