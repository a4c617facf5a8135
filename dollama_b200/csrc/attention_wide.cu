// Flash attention on tcgen05 for wide heads: head_dim 128..512 (multiple of 64) — the SDXL VAE
// mid-block attention (one head, Dh = 512, S = h*w tokens) that the reference runs through its
// general launch_attention (src/kernels/vae_decode.cu:682-683, attention.cuh:53-73).
//
// out = softmax(Q K^T * scale) V with an fp32 online softmax, P kept unnormalised in fp16
// (p = 2^(s c - m c) <= 2^8 under the lazy running max) and the division by the fp32 row sum
// done once on the fp32 accumulator at the end — no S x S score matrix in memory.
//
// One CTA = one (batch, head, 128-query tile, output slice of dv = Dh or Dh / 2 <= 256 columns);
// for Dh = 512 the two slices of a query tile are neighbouring CTAs that each recompute S (the
// K tiles they share come from L2 once).  192 threads, one CTA per SM, all 512 TMEM columns:
//   warps 0..3  softmax: thread r owns query row r (TMEM lane r).  Per 128-key tile j: pass 1
//               reads S_j for the row max (the running max m moves only when a tile's max exceeds
//               it by more than 8 in exp2 units, and then O is rescaled in place), pass 2 writes
//               p = 2^(s c - m c) as fp16 pairs into the first 64 columns of S_j's region, the
//               A operand of the P.V MMA;
//   warp 4      TMA producer: Q once (Dh / 64 chunks of 128 x 64, resident: 128 KB at Dh = 512),
//               then per key tile Dh / 64 K chunks (128 keys x 64 dims) and 4 V chunks (32 keys x
//               dv dims as dv / 64 boxes of 32 x 64) through one ring of 16 KB stages;
//   warp 5      TMEM owner + single-thread MMA issuer: S_j = Q K_j^T (M = 128, N = 128, K = Dh)
//               into region j & 1, O += P_j V_j (M = 128, N = dv, K = 128, P from TMEM, V as an
//               MN-major operand).  Order S_0, S_1, PV_0, S_2, PV_1, ...: S_{j+1} is computed
//               while the softmax of tile j runs (two S regions), and S_{j+2} reuses P_j's region
//               only after PV_j (in-order MMAs).
// TMEM columns: S regions [0,128) and [128,256) (P_j in the first 64 columns of its region),
// O [256, 256 + dv).  No multicast loads.
#include <cuda_fp16.h>

#include "attention.h"
#include "ptx.cuh"

namespace dlm {

namespace {

constexpr int kWQ = 128;           // queries per CTA
constexpr int kWKV = 128;          // keys per tile
constexpr int kWMaxDv = 256;       // output columns per CTA
constexpr int kWStages = 6;
constexpr int kWStageBytes = 16384;
constexpr int kWChunkBytes = kWQ * 64 * 2;  // one 128 x 64 fp16 chunk (Q or K): 16 KB
constexpr int kWVSub = 32 * 64 * 2;         // one 32-key x 64-dim V box: 4 KB
constexpr int kWThreads = 192;
constexpr uint32_t kWTmemCols = 512;

// The ring comes first so that any operand read of a stage stays inside the CTA's shared memory.
constexpr int kWSmemRing = 0;
constexpr int kWSmemQ = kWSmemRing + kWStages * kWStageBytes;   // 96 KB
constexpr int kWSmemBar = kWSmemQ + 8 * kWChunkBytes;           // + 128 KB
constexpr int kWSmem = kWSmemBar + 256 + 1024;
static_assert(kWSmem <= 227 * 1024, "shared memory");

__global__ void __launch_bounds__(kWThreads, 1)
    attn_wide_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnWideParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem + kWSmemRing;
  uint8_t* sQ = smem + kWSmemQ;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWSmemBar);
  uint64_t* q_full = bars;                    // Q loaded
  uint64_t* full = bars + 1;                  // [stages]
  uint64_t* empty = full + kWStages;          // [stages]
  uint64_t* s_full = empty + kWStages;        // [2] S_j ready in region j & 1
  uint64_t* p_full = s_full + 2;              // P_j stored (128 softmax threads)
  uint64_t* o_full = p_full + 1;              // PV_j accumulated into O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nc = p.Dh / 64;                        // K chunks per key tile (and Q chunks)
  const int nsub = p.dv / 64;                      // V boxes per V chunk
  const int n_tiles = (p.Sk + kWKV - 1) / kWKV;
  const int q_tiles = (p.Sq + kWQ - 1) / kWQ;
  int rest = blockIdx.x;
  const int split = rest % p.nsplit;
  rest /= p.nsplit;
  const int q0 = (rest % q_tiles) * kWQ;
  rest /= q_tiles;
  const int h = rest % p.H;
  const int b = rest / p.H;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, kWQ);
    mbar_init(o_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kWTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  griddep_wait();  // q / k / v are written by the previous kernel

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(nc) * kWChunkBytes);
      for (int c = 0; c < nc; ++c) tma_load_4d(sQ + c * kWChunkBytes, &tmQ, q_full, c * 64, h, q0, b);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto next_stage = [&]() -> bool {
        return mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kDevTimeoutProducer);
      };
      auto advance = [&]() {
        if (++stage == kWStages) {
          stage = 0;
          phase ^= 1;
        }
      };
      // the MMA issuer's order: K_0, K_1, then V_j, K_{j+2} for each j
      auto load_k = [&](int j) {
        for (int c = 0; c < nc && ok; ++c) {
          if (!(ok = next_stage())) break;
          mbar_arrive_expect_tx(&full[stage], kWChunkBytes);
          tma_load_4d(ring + stage * kWStageBytes, &tmK, &full[stage], c * 64, h, j * kWKV, b);
          advance();
        }
      };
      auto load_v = [&](int j) {
        for (int vc = 0; vc < 4 && ok; ++vc) {
          if (!(ok = next_stage())) break;
          mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(nsub) * kWVSub);
          for (int i = 0; i < nsub; ++i)
            tma_load_4d(ring + stage * kWStageBytes + i * kWVSub, &tmV, &full[stage],
                        split * p.dv + i * 64, h, j * kWKV + vc * 32, b);
          advance();
        }
      };
      load_k(0);
      if (n_tiles > 1) load_k(1);
      for (int j = 0; j < n_tiles && ok; ++j) {
        load_v(j);
        if (j + 2 < n_tiles) load_k(j + 2);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16_f32(kWQ, kWKV, false);
      const uint32_t idesc_o = idesc_f16_f32(kWQ, p.dv, true);
      int stage = 0;
      uint32_t phase = 0;
      auto take = [&]() -> bool {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kDevTimeoutMma)) return false;
        tc_fence_after();
        return true;
      };
      auto release = [&]() {
        umma_commit(&empty[stage]);
        if (++stage == kWStages) {
          stage = 0;
          phase ^= 1;
        }
      };
      auto issue_s = [&](int j) -> bool {
        const uint32_t d = tbase + (j & 1) * kWKV;
        for (int c = 0; c < nc; ++c) {
          if (!take()) return false;
          const uint32_t q_addr = smem_u32(sQ + c * kWChunkBytes);
          const uint32_t k_addr = smem_u32(ring + stage * kWStageBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ss(d, sw128_desc(q_addr + k * 32, 16, 1024), sw128_desc(k_addr + k * 32, 16, 1024),
                        idesc_s, (c != 0 || k != 0) ? 1u : 0u);
          release();
        }
        umma_commit(&s_full[j & 1]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const uint32_t p_tmem = tbase + (j & 1) * kWKV;
        for (int vc = 0; vc < 4; ++vc) {
          if (!take()) return false;
          const uint32_t v_addr = smem_u32(ring + stage * kWStageBytes);
#pragma unroll
          for (int ks = 0; ks < 2; ++ks)
            umma_f16_ts(tbase + 2 * kWKV, p_tmem + vc * 16 + ks * 8,
                        sw128_desc(v_addr + ks * 2048, kWVSub, 1024), idesc_o,
                        (j != 0 || vc != 0 || ks != 0) ? 1u : 0u);
          release();
        }
        umma_commit(o_full);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kDevTimeoutMma);
      if (ok) ok = issue_s(0);
      if (ok && n_tiles > 1) ok = issue_s(1);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (!(ok = mbar_wait(p_full, j & 1, abort_flag, p.status, kDevTimeoutMma))) break;
        tc_fence_after();
        ok = issue_pv(j);
        if (ok && j + 2 < n_tiles) ok = issue_s(j + 2);
      }
      griddep_launch_dependents();
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int row = warp * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t to = tbase + lane_off + 2 * kWKV;
    const float c = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.status, kDevTimeoutSoftmax));
    };
    for (int j = 0; j < n_tiles && ok; ++j) {
      const uint32_t ts = tbase + lane_off + (j & 1) * kWKV;
      if (!(ok = wwait(&s_full[j & 1], (j >> 1) & 1))) break;
      tc_fence_after();
      const int valid = p.Sk - j * kWKV;
      const bool full_tile = valid >= kWKV;
      // pass 1: the tile's row max
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
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
      float m_new = m_run, alpha = 1.0f;
      if (j == 0) {
        m_new = mx;
      } else if ((mx - m_run) * c > 8.0f) {
        m_new = mx;
        alpha = fast_exp2((m_run - mx) * c);
      }
      // pass 2: p = 2^(s c - m c) as fp16 pairs into the region's first 64 columns (this lane has
      // read them already), fp32 row sum
      const float mc = m_new * c;
      const uint64_t c2 = f2_pack(c, c), nmc2 = f2_pack(-mc, -mc);
      uint64_t sumA = f2_pack(0.0f, 0.0f), sumB = sumA;
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(ts + cc * 32, ra);
        tmem_ld_32x32b_x32(ts + cc * 32 + 32, rb);
        tmem_ld_wait();
        uint32_t pp[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t* r = half ? rb : ra;
          const int col0 = (cc + half) * 32;
#pragma unroll
          for (int q = 0; q < 32; q += 2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(r[q]), __uint_as_float(r[q + 1])), c2, nmc2), x0, x1);
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
        tmem_st_32x32b_x32(ts + (cc >> 1) * 32, pp);
      }
      tmem_st_wait();
      if (j >= 1) {
        // PV_{j-1} has completed: O may be rescaled before PV_j adds into it
        if (!(ok = wwait(o_full, (j - 1) & 1))) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
          const uint64_t a2 = f2_pack(alpha, alpha), z2 = f2_pack(0.0f, 0.0f);
          for (int oc = 0; oc < p.dv; oc += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(to + oc, r);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(r[q]), __uint_as_float(r[q + 1])), a2, z2), x0, x1);
              r[q] = __float_as_uint(x0);
              r[q + 1] = __float_as_uint(x1);
            }
            tmem_st_32x32b_x32(to + oc, r);
          }
          tmem_st_wait();
        }
      }
      float s0, s1, s2, s3;
      f2_unpack(sumA, s0, s1);
      f2_unpack(sumB, s2, s3);
      tc_fence_before();
      mbar_arrive(p_full);
      l_run = fmaf(l_run, alpha, (s0 + s1) + (s2 + s3));
      m_run = m_new;
    }
    if (ok && n_tiles > 0) ok = wwait(o_full, (n_tiles - 1) & 1);
    if (ok) {
      tc_fence_after();
      const int qrow = q0 + row;
      const float inv = 1.0f / l_run;
      __half* dst = p.out + static_cast<size_t>(b) * p.o_sb + static_cast<size_t>(h) * p.o_sh +
                    static_cast<size_t>(qrow) * p.o_ss + static_cast<size_t>(split) * p.dv;
      for (int oc = 0; oc < p.dv; oc += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(to + oc, r);
        tmem_ld_wait();
        if (qrow < p.Sq) {
#pragma unroll
          for (int q = 0; q < 32; q += 8) {
            uint4 v;
            v.x = pack_half2(__uint_as_float(r[q]) * inv, __uint_as_float(r[q + 1]) * inv);
            v.y = pack_half2(__uint_as_float(r[q + 2]) * inv, __uint_as_float(r[q + 3]) * inv);
            v.z = pack_half2(__uint_as_float(r[q + 4]) * inv, __uint_as_float(r[q + 5]) * inv);
            v.w = pack_half2(__uint_as_float(r[q + 6]) * inv, __uint_as_float(r[q + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + oc + q) = v;
          }
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_sleep(200000);
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kWTmemCols);
  }
}

bool make_wide_map(CUtensorMap* m, const AttnTensor& t, int Dh, int B, int H, int S, int rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(Dh), static_cast<uint64_t>(H),
                            static_cast<uint64_t>(S), static_cast<uint64_t>(B)};
  const uint64_t st[3] = {static_cast<uint64_t>(t.sh) * 2, static_cast<uint64_t>(t.ss) * 2,
                          static_cast<uint64_t>(t.sb) * 2};
  const uint32_t box[4] = {64, 1, static_cast<uint32_t>(rows), 1};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, t.ptr, dims, st, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

bool wide_stride_ok(const AttnTensor& t) {
  return (reinterpret_cast<uintptr_t>(t.ptr) & 15) == 0 && t.sh % 8 == 0 && t.ss % 8 == 0 &&
         t.sb % 8 == 0 && t.sh > 0 && t.ss > 0 && t.sb > 0;
}

}  // namespace

int attn_wide_plan(AttnWideOp* op, int B, int H, int Sq, int Sk, int Dh, float scale,
                   const AttnTensor& q, const AttnTensor& k, const AttnTensor& v,
                   const AttnTensor& o) {
  DLM_REQUIRE(op != nullptr, DLM_ERR_INVALID, "attention: null op");
  DLM_REQUIRE(B > 0 && H > 0 && Sq > 0 && Sk > 0, DLM_ERR_INVALID, "attention: empty problem");
  DLM_REQUIRE(Dh % 64 == 0 && Dh >= 128 && Dh <= 512, DLM_ERR_UNSUPPORTED,
              "attention: head_dim %d (wide heads: a multiple of 64 in [128, 512])", Dh);
  DLM_REQUIRE(q.ptr && k.ptr && v.ptr && o.ptr, DLM_ERR_INVALID, "attention: null tensor");
  DLM_REQUIRE(wide_stride_ok(q) && wide_stride_ok(k) && wide_stride_ok(v) && wide_stride_ok(o),
              DLM_ERR_INVALID, "attention: tensors must be 16-byte aligned with strides %% 8 == 0");
  std::memset(op, 0, sizeof(*op));
  if (!make_wide_map(&op->tmQ, q, Dh, B, H, Sq, kWQ)) return DLM_ERR_CUDA;
  if (!make_wide_map(&op->tmK, k, Dh, B, H, Sk, kWKV)) return DLM_ERR_CUDA;
  if (!make_wide_map(&op->tmV, v, Dh, B, H, Sk, 32)) return DLM_ERR_CUDA;
  AttnWideParams& p = op->p;
  p.B = B;
  p.H = H;
  p.Sq = Sq;
  p.Sk = Sk;
  p.Dh = Dh;
  p.nsplit = Dh > kWMaxDv ? 2 : 1;
  p.dv = Dh / p.nsplit;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = const_cast<__half*>(o.ptr);
  p.o_sb = o.sb;
  p.o_sh = o.sh;
  p.o_ss = o.ss;
  p.status = device_status_ptr();
  const long long grid = static_cast<long long>(B) * H * ((Sq + kWQ - 1) / kWQ) * p.nsplit;
  DLM_REQUIRE(grid < (1ll << 31), DLM_ERR_INVALID, "attention: too many query tiles");
  op->grid = static_cast<int>(grid);
  return DLM_OK;
}

int attn_wide_launch(const AttnWideOp& op, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    DLM_CHECK_CUDA(cudaFuncSetAttribute(attn_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kWSmem));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(op.grid, 1, 1);
  cfg.blockDim = dim3(kWThreads, 1, 1);
  cfg.dynamicSmemBytes = kWSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  DLM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn_wide_kernel, op.tmQ, op.tmK, op.tmV, op.p));
  return DLM_OK;
}

}  // namespace dlm
