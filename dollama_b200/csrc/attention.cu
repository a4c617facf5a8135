// Flash attention on tcgen05 for head_dim 64 (SDXL self / cross attention).
//
// Replaces launch_attention / launch_attention_fast (reference src/kernels/attention.cuh:53-73,
// attention.cu:393, attention_fast.cu:58): out = softmax(Q K^T * scale) V with an fp32 online
// softmax and P rounded to fp16 for the P.V product (as attention_fast.cu:238 does).
//
// One CTA = one (batch, head, 128-query tile); 192 threads:
//   warps 0..3  softmax: thread r owns query row r (TMEM lane r).  Per 128-key tile j it reads
//               S_j from TMEM (two passes of 4 x 32 columns: row max, then exp2 / row sum),
//               writes P_j (fp16) into a 128-byte-swizzled K-major shared tile, then folds the
//               previous tile's P.V result O_{j-1} (TMEM, 64 columns) into its fp32 register
//               accumulator with the running rescale;
//   warp 4      TMA producer: Q once, then K_j / V_j into a KV_STAGES ring;
//   warp 5      TMEM owner + single-thread MMA issuer: S_j = Q K_j^T (M=128, N=128, K=64) into
//               S[j%2]; O_j = P_j V_j (M=128, N=64, K=128, V as an MN-major operand) into O[j%2].
// S and O are double-buffered in TMEM (2x128 + 2x64 of 512 columns) so that S_{j+1} and
// P_j V_j run on the tensor core while the softmax warps work on tile j.
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

constexpr int kQ = 128;        // queries per CTA
constexpr int kKV = 128;       // keys per tile
constexpr int kD = 64;         // head dim
constexpr int kKVStages = 3;
constexpr int kAttnThreads = 192;
constexpr int kTileBytes = kQ * kD * 2;          // 16 KB (Q, K or V tile)
constexpr int kPBytes = kQ * kKV * 2;            // 32 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO0 = 256;     // S[b] at 128*b, O[b] at 256 + 64*b

constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + kTileBytes;
constexpr int kSmemV = kSmemK + kKVStages * kTileBytes;
constexpr int kSmemP = kSmemV + kKVStages * kTileBytes;
constexpr int kSmemBar = kSmemP + 2 * kPBytes;
constexpr int kAttnSmem = kSmemBar + 256 + 1024;

__device__ __forceinline__ void store_p_chunk(uint8_t* pbuf, int row, int chunk32,
                                              const uint32_t (&h)[16]) {
  // keys [32*chunk32, +32) of `row`: four 16-byte chunks, 128B-swizzled K-major layout with
  // two 64-key column blocks of 16 KB each.
  const int blk = chunk32 >> 1;
  uint8_t* base = pbuf + blk * (kQ * 128) + row * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c16 = ((chunk32 & 1) * 4 + i) ^ (row & 7);
    *reinterpret_cast<uint4*>(base + c16 * 16) =
        make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
  }
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + kSmemQ;
  uint8_t* sK = smem + kSmemK;
  uint8_t* sV = smem + kSmemV;
  uint8_t* sP = smem + kSmemP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kKVStages;
  uint64_t* kv_empty = v_full + kKVStages;
  uint64_t* s_full = kv_empty + kKVStages;  // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_full = p_full + 2;            // [2]
  uint64_t* o_empty = o_full + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q_tiles = (p.Sq + kQ - 1) / kQ;
  const int qt = blockIdx.x % q_tiles;
  const int bh = blockIdx.x / q_tiles;
  const int h = bh % p.H;
  const int b = bh / p.H;
  const int q0 = qt * kQ;
  const int n_tiles = (p.Sk + kKV - 1) / kKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kQ);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], kQ);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tmQ, q_full, 0, h, q0, b);
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < n_tiles; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer)) break;
        mbar_arrive_expect_tx(&k_full[stage], kTileBytes);
        tma_load_4d(sK + stage * kTileBytes, &tmK, &k_full[stage], 0, h, j * kKV, b);
        mbar_arrive_expect_tx(&v_full[stage], kTileBytes);
        tma_load_4d(sV + stage * kTileBytes, &tmV, &v_full[stage], 0, h, j * kKV, b);
        if (++stage == kKVStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(kQ, kKV, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(kQ, kD, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kDevTimeoutMma);
      // S_j for j = 0, 1
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKVStages;
        const uint32_t ph = (j / kKVStages) & 1;
        if (!mbar_wait(&k_full[st], ph, abort_flag, p.status, kDevTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * kTileBytes);
        const uint32_t d = tbase + kColS0 + (j & 1) * kKV;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          umma_f16_ss(d, sw128_desc(q_addr + k * 32, 16, 1024), sw128_desc(k_addr + k * 32, 16, 1024),
                      idesc_s, k != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_tiles > 1) ok = issue_s(1);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j % kKVStages;
        const uint32_t ph = (j / kKVStages) & 1;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutMma)) break;
        if (!mbar_wait(&v_full[st], ph, abort_flag, p.status, kDevTimeoutMma)) break;
        if (j >= 2 &&
            !mbar_wait(&o_empty[j & 1], ((j - 2) >> 1) & 1, abort_flag, p.status, kDevTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP + (j & 1) * kPBytes);
        const uint32_t v_addr = smem_u32(sV + st * kTileBytes);
        const uint32_t d = tbase + kColO0 + (j & 1) * kD;
#pragma unroll
        for (int ks = 0; ks < kKV / 16; ++ks) {
          const uint64_t ad = sw128_desc(p_addr + (ks >> 2) * (kQ * 128) + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(v_addr + ks * 2048, 1024, 1024);
          umma_f16_ss(d, ad, bd, idesc_o, ks != 0 ? 1u : 0u);
        }
        umma_commit(&o_full[j & 1]);
        umma_commit(&kv_empty[st]);
        if (j + 2 < n_tiles) ok = issue_s(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int row = warp * 32 + lane;  // TMEM lane == query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float c = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.0f, alpha_prev = 1.0f;
    float acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) acc[d] = 0.0f;
    bool ok = true;

    auto fold_o = [&](int j, float alpha) -> bool {
      if (!mbar_wait(&o_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax))
        return false;
      tc_fence_after();
      const uint32_t ta = tbase + lane_off + kColO0 + (j & 1) * kD;
      uint32_t r[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld_32x32b_x32(ta + half * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 32; ++q) acc[half * 32 + q] = acc[half * 32 + q] * alpha + __uint_as_float(r[q]);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[j & 1]);
      return true;
    };

    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, abort_flag, p.status, kDevTimeoutSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tbase + lane_off + kColS0 + (j & 1) * kKV;
      const int valid = p.Sk - j * kKV;  // keys of this tile that exist (may exceed 128)
      // pass 1: row max
      float mx = m_run;
      uint32_t r[32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        tmem_ld_32x32b_x32(ts + cc * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const float s = (cc * 32 + q < valid) ? __uint_as_float(r[q]) : -INFINITY;
          mx = fmaxf(mx, s);
        }
      }
      const float alpha = fast_exp2((m_run - mx) * c);  // m_run = -inf on the first tile -> 0
      const float mc = mx * c;
      // pass 2: p = exp2(s*c - m*c), row sum, fp16 P into shared memory
      float sum = 0.0f;
      uint8_t* pbuf = sP + (j & 1) * kPBytes;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        tmem_ld_32x32b_x32(ts + cc * 32, r);
        tmem_ld_wait();
        uint32_t hp[16];
#pragma unroll
        for (int q = 0; q < 32; q += 2) {
          const float s0 = (cc * 32 + q < valid) ? __uint_as_float(r[q]) : -INFINITY;
          const float s1 = (cc * 32 + q + 1 < valid) ? __uint_as_float(r[q + 1]) : -INFINITY;
          const float e0 = fast_exp2(fmaf(s0, c, -mc));
          const float e1 = fast_exp2(fmaf(s1, c, -mc));
          const __half2 hh = __floats2half2_rn(e0, e1);
          const float2 back = __half22float2(hh);
          sum += back.x + back.y;  // the sum matches the fp16 P that multiplies V
          hp[q >> 1] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        store_p_chunk(pbuf, row, cc, hp);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      l_run = l_run * alpha + sum;
      m_run = mx;
      if (j >= 1) {
        if (!fold_o(j - 1, alpha_prev)) {
          ok = false;
          break;
        }
      }
      alpha_prev = alpha;
    }
    if (ok && n_tiles > 0) ok = fold_o(n_tiles - 1, alpha_prev);
    if (ok && q0 + row < p.Sq) {
      const float inv = 1.0f / l_run;
      __half* dst = p.out + static_cast<size_t>(b) * p.o_sb + static_cast<size_t>(h) * p.o_sh +
                    static_cast<size_t>(q0 + row) * p.o_ss;
#pragma unroll
      for (int d = 0; d < kD; d += 8) {
        uint4 v;
        v.x = pack_half2(acc[d] * inv, acc[d + 1] * inv);
        v.y = pack_half2(acc[d + 2] * inv, acc[d + 3] * inv);
        v.z = pack_half2(acc[d + 4] * inv, acc[d + 5] * inv);
        v.w = pack_half2(acc[d + 6] * inv, acc[d + 7] * inv);
        *reinterpret_cast<uint4*>(dst + d) = v;
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 5) {
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

int attn_plan(AttnOp* op, int B, int H, int Sq, int Sk, int Dh, float scale, const AttnTensor& q,
              const AttnTensor& k, const AttnTensor& v, const AttnTensor& o) {
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
  op->grid = B * H * ((Sq + kQ - 1) / kQ);
  return DLM_OK;
}

int attn_prepare_kernels() {
  DLM_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kAttnSmem));
  return DLM_OK;
}

int attn_launch(const AttnOp& op, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    DLM_CHECK_CUDA(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kAttnSmem));
    attr_set[dev] = true;
  }
  attn_fwd_kernel<<<op.grid, kAttnThreads, kAttnSmem, s>>>(op.tmQ, op.tmK, op.tmV, op.p);
  DLM_CHECK_CUDA(cudaGetLastError());
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
  dlm::AttnOp op;
  int rc = dlm::attn_plan(&op, B, H, Sq, Sk, Dh, scale, bhsd(q, Sq), bhsd(k, Sk), bhsd(v, Sk),
                          bhsd(out, Sq));
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
  dlm::AttnOp op;
  int rc = dlm::attn_plan(&op, B, H, Sq, Sk, Dh, scale, tok(q, ldq, Sq), tok(k, ldk, Sk),
                          tok(v, ldv, Sk), tok(out, ldo, Sq));
  if (rc != DLM_OK) return rc;
  return dlm::attn_launch(op, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
