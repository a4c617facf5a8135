// Host side of the tcgen05 GEMM: tile-width choice, tensor-map encoding, launch, and the
// GEMM entry points of the C ABI.
#include <cstring>

#include "gemm.h"
#include "gemm_launch.cuh"
#include "ops.h"

namespace dlm {

namespace {

// Tile choice, calibrated on B200 sweeps of the UNet shapes (single CTA vs CTA pair, every N
// tile).  The single-CTA kernel is bound by how fast TMA can pull operands from L2 into one SM
// (about 70-85 B/clock with every SM loading), which narrow tiles hit first; its relative cost per
// k-block and unit of N is modelled as max(BN, (128 + BN) / 2) + 24 per tile, times the number of
// waves.  The CTA pair halves B traffic per SM but measured faster only for wide-N problems with
// few row tiles (N >= 2560, M <= 4096, BN = 256: +5-7%), so it is used there alone.
double tile_cost(int bn) {
  const double mma = bn;
  const double smem = 0.5 * (128 + bn);
  return (mma > smem ? mma : smem) + 24.0;
}

// Largest number of CTA pairs of gemm_tc2_kernel<BN, *> co-resident on the current device (clusters
// are placed within a GPC, so an SM without a free partner in its GPC cannot host a pair).
template <int BN>
int max_pairs_bn() {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * num_sms(), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = gemm2_smem_bytes(BN);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaFuncSetAttribute(gemm_tc2_kernel<BN, kEpiDyn>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       gemm2_smem_bytes(BN));
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<BN, kEpiDyn>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = num_sms() / 2;
  }
  return n;
}

int max_pairs(int bn) {
  static int cache[64][5] = {{0}};
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = bn == 256 ? 0 : bn == 192 ? 1 : bn == 160 ? 2 : bn == 224 ? 4 : 3;
  if (dev < 0 || dev >= 64) return num_sms() / 2;
  if (cache[dev][slot] == 0) {
    cache[dev][slot] = bn == 256 ? max_pairs_bn<256>() : bn == 224 ? max_pairs_bn<224>()
                     : bn == 192 ? max_pairs_bn<192>() : bn == 160 ? max_pairs_bn<160>()
                     : max_pairs_bn<128>();
  }
  return cache[dev][slot];
}

// Chooses single-CTA vs CTA-pair and the N tile.  Dense linears (conv == false) with more than
// one row tile run on CTA pairs, whose two-k-block stages keep the issuing thread ahead of the
// tensor pipe; the N tile minimises waves x measured clocks per k-block (B200, UNet shapes:
// ~590 for a 256 x 160 pair tile, ~600 for 256 x 224, ~634 for 256 x 256; 224 wins where it
// rounds the tile count under a whole number of waves that 256 exceeds, e.g. the 32^2 level's
// q|k|v 2048 x 3840 x 1280: 19.0 -> 17.5 us).  Implicit-GEMM convolutions measured
// faster on single CTAs (their 4D im2col boxes) and keep the single-CTA cost model.
void pick_tile(int M, int N, bool conv, int force_bn, int force_mode, int* bn_out, bool* pair_out) {
  static const int single[] = {256, 192, 160, 128, 64};
  static const int paired[] = {256, 224, 192, 160, 128};
  const int sms = num_sms();
  const bool want_pair = force_mode == 2 || (force_mode == 0 && !conv && M > kGemmBM);
  if (want_pair && M > kGemmBM) {
    int bn = force_bn;
    if (bn == 0) {
      const long mt2 = (M + 2 * kGemmBM - 1) / (2 * kGemmBM);
      double best = 1e30;
      for (int c : {256, 224, 160}) {
        const long tiles = mt2 * ((N + c - 1) / c);
        const long pairs = max_pairs(c);
        const double clk = c == 256 ? 634.0 : c == 224 ? 600.0 : 590.0;
        const double cost = static_cast<double>((tiles + pairs - 1) / pairs) * clk;
        if (cost < best - 1e-9) {
          best = cost;
          bn = c;
        }
      }
    }
    bool ok = false;
    for (int c : paired) ok = ok || c == bn;
    if (ok) {
      *bn_out = bn;
      *pair_out = true;
      return;
    }
  }
  const long mt = (M + kGemmBM - 1) / kGemmBM;
  double best = 1e30;
  int bn_best = 128;
  for (int bn : single) {
    if (force_bn && bn != force_bn) continue;
    const long tiles = mt * ((N + bn - 1) / bn);
    const double c = ((tiles + sms - 1) / sms) * tile_cost(bn);
    if (c < best - 1e-9) {
      best = c;
      bn_best = bn;
    }
  }
  *bn_out = bn_best;
  *pair_out = false;
}

int g_force_mode = 0;  // test hook: 0 auto, 1 single CTA, 2 CTA pair, 3 stream-K
int g_force_bn = 0;    // test hook: forced N tile (0 = cost model)

// Stream-K choice (single-CTA kernel over all SMs).  Only on request (tile mode 3): B200 sweeps
// of the UNet shapes (M = 2048 / 8192 linears, long-K convs) measured the single-CTA stream-K
// launch 1.3-3x slower than whole tiles, because with every SM loading 128 x 256 tiles the
// aggregate L2 -> SM traffic (about 9 TB/s here) rather than the idle SMs bounds these launches;
// splitting K does not reduce that traffic, larger (CTA-pair) tiles do.  Returns the N tile for
// stream-K, or 0.
int pick_stream_k(long m_tiles, int N, int num_kb, int bn, bool pair, const GemmEpilogue& e,
                  int force_mode, int force_bn) {
  const int sms = num_sms();
  if (e.sk_ws == nullptr) return 0;
  auto fits = [&](int b) {
    return static_cast<size_t>(sms) * kGemmBM * b * 4 + gemm_sk_flag_bytes() <= e.sk_ws_bytes;
  };
  int best = 0;
  long best_units = 0;
  for (int b : {256, 192, 160, 128}) {
    if (force_bn && b != force_bn) continue;
    const long units = (m_tiles * ((N + b - 1) / b) * num_kb + sms - 1) / sms;
    if (best == 0 || units < best_units) {
      best = b;
      best_units = units;
    }
  }
  if (best == 0 || !fits(best)) return 0;
  (void)bn;
  (void)pair;
  (void)best_units;
  return force_mode == 3 ? best : 0;
}

bool bn_supported(int bn, bool pair) {
  if (pair) return bn == 256 || bn == 224 || bn == 192 || bn == 160 || bn == 128;
  return bn == 256 || bn == 192 || bn == 160 || bn == 128 || bn == 64;
}

// Output map for the staged epilogue: boxes of 32 rows x 32 columns (64-byte swizzle), or
// 32 rows x 16 columns (32-byte swizzle) for GEGLU's half-width output.
bool make_out_map(CUtensorMap* m, const __half* C, int M, int N, int ldc, unsigned flags) {
  if (flags & kEpiOutF32) {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 4};
    const uint32_t box[2] = {16u, 32u};
    return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_64B);
  }
  const bool geglu = (flags & DLM_EPI_GEGLU) != 0;
  const uint64_t cols = geglu ? N / 2 : N;
  const uint64_t dims[2] = {cols, static_cast<uint64_t>(M)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 2};
  const uint32_t box[2] = {geglu ? 16u : 32u, 32u};
  return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, C, dims, strides, box,
                     geglu ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B);
}

void fill_epilogue(GemmParams& p, const GemmEpilogue& e, int N) {
  p.flags = e.flags;
  p.alpha = e.alpha;
  p.resid_scale = e.resid_scale;
  p.bias = e.bias;
  p.bias2d = e.bias2d;
  p.rows_per_img = e.rows_per_img > 0 ? e.rows_per_img : 1;
  p.ldb2 = e.ldb2 > 0 ? e.ldb2 : N;
  p.resid = e.resid;
  p.ldr = e.ldr;
  p.stats_out = e.stats_out;
  p.stats_in = e.stats_in;
  p.stats_in_parts = e.stats_in_parts;
  p.stats_in_tile = e.stats_in_tile;
  p.ln_C = e.ln_C;
  p.ln_eps = e.ln_eps;
  p.ln_u = e.ln_u;
  p.ln_v = e.ln_v;
}

int check_epilogue(const GemmEpilogue& e, int N, __half* C, int ldc) {
  DLM_REQUIRE(C != nullptr, DLM_ERR_INVALID, "gemm: null output");
  DLM_REQUIRE((reinterpret_cast<uintptr_t>(C) & 15) == 0 && ldc % 8 == 0, DLM_ERR_INVALID,
              "gemm: output must be 16-byte aligned with ldc %% 8 == 0 (ldc=%d)", ldc);
  const int out_cols = (e.flags & DLM_EPI_GEGLU) ? N / 2 : N;
  DLM_REQUIRE(ldc >= out_cols, DLM_ERR_INVALID, "gemm: ldc=%d < output columns %d", ldc, out_cols);
  if (e.flags & DLM_EPI_RESID)
    DLM_REQUIRE(e.ldr >= N, DLM_ERR_INVALID, "gemm: ldr=%d < N=%d", e.ldr, N);
  if (e.flags & DLM_EPI_BIAS)
    DLM_REQUIRE(e.bias != nullptr && (reinterpret_cast<uintptr_t>(e.bias) & 15) == 0,
                DLM_ERR_INVALID, "gemm: bias must be non-null and 16-byte aligned");
  if (e.flags & DLM_EPI_BIAS2D)
    DLM_REQUIRE(e.bias2d != nullptr && (reinterpret_cast<uintptr_t>(e.bias2d) & 15) == 0,
                DLM_ERR_INVALID, "gemm: bias2d must be non-null and 16-byte aligned");
  if (e.flags & DLM_EPI_RESID)
    DLM_REQUIRE(e.resid != nullptr && (reinterpret_cast<uintptr_t>(e.resid) & 15) == 0 &&
                    e.ldr % 8 == 0,
                DLM_ERR_INVALID, "gemm: residual must be 16-byte aligned with ldr %% 8 == 0");
  if (e.flags & DLM_EPI_GEGLU)
    DLM_REQUIRE(!(e.flags & DLM_EPI_RESID) && !(e.flags & kEpiRowStats) && N % 64 == 0,
                DLM_ERR_INVALID, "gemm: GEGLU needs N %% 64 == 0, no residual, no row statistics");
  if (e.flags & kEpiRowStats)
    DLM_REQUIRE(e.stats_out != nullptr && !(e.flags & kEpiOutF32), DLM_ERR_INVALID,
                "gemm: row statistics need a buffer and an fp16 output");
  if (e.flags & kEpiOutF32)
    DLM_REQUIRE(!(e.flags & DLM_EPI_GEGLU) && ldc % 4 == 0, DLM_ERR_INVALID,
                "gemm: fp32 output needs ldc %% 4 == 0 and no GEGLU");
  if (e.flags & kEpiResidF32)
    DLM_REQUIRE((e.flags & DLM_EPI_RESID) && e.ldr % 4 == 0, DLM_ERR_INVALID,
                "gemm: fp32 residual needs ldr %% 4 == 0");
  if (e.flags & kEpiLnFold)
    DLM_REQUIRE(e.stats_in && e.ln_u && e.ln_v && e.stats_in_parts > 0 && e.stats_in_tile > 0 &&
                    e.ln_C > 0 && (reinterpret_cast<uintptr_t>(e.ln_u) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(e.ln_v) & 15) == 0,
                DLM_ERR_INVALID, "gemm: LayerNorm fold needs statistics and 16-byte aligned u / v");
  return DLM_OK;
}

// Grid of a planned op: whole tiles (at most one CTA / pair per SM), or stream-K over every SM
// with the workspace's flag head and partial slots.
void set_grid(GemmOp* op, bool stream_k, const GemmEpilogue& e) {
  GemmParams& p = op->p;
  if (stream_k) {
    p.sk_ctas = num_sms();
    p.sk_flags = static_cast<int*>(e.sk_ws);
    p.sk_ws = reinterpret_cast<float*>(static_cast<char*>(e.sk_ws) + gemm_sk_flag_bytes());
    op->grid = p.sk_ctas;
    return;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int slots = op->pair ? max_pairs(op->bn) : num_sms();
  op->grid = (tiles < slots ? tiles : slots) * (op->pair ? 2 : 1);
}

}  // namespace

size_t gemm_sk_flag_bytes() { return ((static_cast<size_t>(num_sms()) * 4 + 255) / 256) * 256; }
size_t gemm_sk_workspace_bytes() {
  return gemm_sk_flag_bytes() + static_cast<size_t>(num_sms()) * kGemmBM * 256 * 4;
}

int gemm_plan_dense(GemmOp* op, const __half* A, int lda, const __half* W, int M, int N, int K,
                    __half* C, int ldc, const GemmEpilogue& epi, int force_bn, int ldw) {
  if (ldw == 0) ldw = K;
  DLM_REQUIRE(ldw >= K && ldw % 8 == 0, DLM_ERR_INVALID, "gemm: ldw=%d must be >= K and a multiple of 8", ldw);
  DLM_REQUIRE(op != nullptr && A != nullptr && W != nullptr, DLM_ERR_INVALID,
              "gemm: null operand");
  DLM_REQUIRE(M > 0 && N > 0 && K > 0, DLM_ERR_INVALID, "gemm: empty problem");
  DLM_REQUIRE(N % 32 == 0, DLM_ERR_INVALID, "gemm: N=%d must be a multiple of 32", N);
  DLM_REQUIRE(K % 8 == 0 && lda % 8 == 0 && lda >= K, DLM_ERR_INVALID,
              "gemm: K=%d and lda=%d must be multiples of 8 (16-byte rows)", K, lda);
  DLM_REQUIRE((reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(W) & 15) == 0,
              DLM_ERR_INVALID, "gemm: operands must be 16-byte aligned");
  int rc = check_epilogue(epi, N, C, ldc);
  if (rc != DLM_OK) return rc;
  int bn = 0;
  bool pair = false;
  pick_tile(M, N, false, force_bn ? force_bn : g_force_bn, g_force_mode, &bn, &pair);
  const int sk_bn = pick_stream_k((M + kGemmBM - 1) / kGemmBM, N, (K + kGemmBK - 1) / kGemmBK, bn,
                                  pair, epi, g_force_mode, force_bn ? force_bn : g_force_bn);
  if (sk_bn) {
    bn = sk_bn;
    pair = false;
  }
  DLM_REQUIRE(bn_supported(bn, pair), DLM_ERR_INVALID, "gemm: unsupported tile width %d", bn);
  std::memset(op, 0, sizeof(*op));
  if (!tmap_2d_f16(&op->tmA[0], A, M, K, lda, kGemmBM, kGemmBK)) return DLM_ERR_CUDA;
  op->tmA[1] = op->tmA[0];
  op->tmA[2] = op->tmA[0];
  if (!tmap_2d_f16(&op->tmB, W, N, K, ldw, pair ? bn / 2 : bn, kGemmBK)) return DLM_ERR_CUDA;
  if (!make_out_map(&op->tmC, C, M, N, ldc, epi.flags)) return DLM_ERR_CUDA;
  GemmParams& p = op->p;
  p.M = M;
  p.N = N;
  p.num_kb = (K + kGemmBK - 1) / kGemmBK;
  p.m_tiles = (M + (pair ? 2 : 1) * kGemmBM - 1) / ((pair ? 2 : 1) * kGemmBM);
  p.n_tiles = (N + bn - 1) / bn;
  p.stats_ld = p.n_tiles;
  p.amode = 0;
  p.out = C;
  p.ldo = ldc;
  fill_epilogue(p, epi, p.N);
  p.status = device_status_ptr();
  op->bn = bn;
  op->pair = pair;
  op->k_true = K;
  set_grid(op, sk_bn != 0, epi);
  return DLM_OK;
}

int gemm_plan_conv(GemmOp* op, int Nb, int oH, int oW, const ConvSource* srcs, int nsrc,
                   const __half* W, int Cout, __half* C, int ldc, const GemmEpilogue& epi,
                   int force_bn) {
  DLM_REQUIRE(op != nullptr && srcs != nullptr && W != nullptr, DLM_ERR_INVALID,
              "conv: null operand");
  DLM_REQUIRE(nsrc >= 1 && nsrc <= 3, DLM_ERR_INVALID, "conv: 1..3 K segments (got %d)", nsrc);
  DLM_REQUIRE(Nb > 0 && oH > 0 && oW > 0 && Cout > 0, DLM_ERR_INVALID, "conv: empty problem");
  DLM_REQUIRE(Cout % 32 == 0, DLM_ERR_INVALID, "conv: Cout=%d must be a multiple of 32", Cout);
  const int bw = oW < 128 ? oW : 128;
  const int bh = 128 / bw;
  DLM_REQUIRE(128 % bw == 0 && oW % bw == 0 && oH % bh == 0, DLM_ERR_INVALID,
              "conv: output %dx%d cannot be tiled by 128-pixel boxes", oH, oW);
  int rc = check_epilogue(epi, Cout, C, ldc);
  if (rc != DLM_OK) return rc;
  const int M = Nb * oH * oW;
  int bn = 0;
  bool pair = false;
  pick_tile(M, Cout, true, force_bn ? force_bn : g_force_bn, g_force_mode, &bn, &pair);
  long ktot_blocks = 0;
  for (int s = 0; s < nsrc; ++s) ktot_blocks += static_cast<long>(srcs[s].kind == 1 ? 1 : 9) * (srcs[s].C / 64);
  const int sk_bn = pick_stream_k(M / kGemmBM, Cout, static_cast<int>(ktot_blocks), bn, pair, epi,
                                  g_force_mode, force_bn ? force_bn : g_force_bn);
  if (sk_bn) {
    bn = sk_bn;
    pair = false;
  }
  DLM_REQUIRE(bn_supported(bn, pair), DLM_ERR_INVALID, "conv: unsupported tile width %d", bn);
  std::memset(op, 0, sizeof(*op));
  GemmParams& p = op->p;
  long ktot = 0;
  for (int s = 0; s < nsrc; ++s) {
    const ConvSource& cs = srcs[s];
    DLM_REQUIRE(cs.ptr != nullptr && (reinterpret_cast<uintptr_t>(cs.ptr) & 15) == 0,
                DLM_ERR_INVALID, "conv: source %d null or misaligned", s);
    DLM_REQUIRE(cs.C > 0 && cs.C % 64 == 0, DLM_ERR_INVALID,
                "conv: source %d channels %d must be a multiple of 64", s, cs.C);
    DLM_REQUIRE(cs.kind >= 0 && cs.kind <= 2, DLM_ERR_INVALID, "conv: bad segment kind");
    const uint64_t c = cs.C;
    if (cs.kind == 2) {
      const uint64_t dims[5] = {c, (uint64_t)oW, (uint64_t)oH, (uint64_t)Nb, 4};
      const uint64_t st[4] = {c * 2, c * oW * 2, c * oW * oH * 2, c * oW * oH * Nb * 2};
      const uint32_t box[5] = {64, (uint32_t)bw, (uint32_t)bh, 1, 1};
      if (!encode_tmap(&op->tmA[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, cs.ptr, dims, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B))
        return DLM_ERR_CUDA;
    } else {
      const uint64_t dims[4] = {c, (uint64_t)oW, (uint64_t)oH, (uint64_t)Nb};
      const uint64_t st[3] = {c * 2, c * oW * 2, c * oW * oH * 2};
      const uint32_t box[4] = {64, (uint32_t)bw, (uint32_t)bh, 1};
      if (!encode_tmap(&op->tmA[s], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, cs.ptr, dims, st, box,
                       CU_TENSOR_MAP_SWIZZLE_128B))
        return DLM_ERR_CUDA;
    }
    p.seg[s].map = s;
    p.seg[s].kind = cs.kind;
    p.seg[s].cblocks = cs.C / 64;
    ktot += static_cast<long>(cs.kind == 1 ? 1 : 9) * cs.C;
  }
  for (int s = nsrc; s < 3; ++s) op->tmA[s] = op->tmA[0];
  if (!tmap_2d_f16(&op->tmB, W, Cout, ktot, ktot, pair ? bn / 2 : bn, kGemmBK)) return DLM_ERR_CUDA;
  if (!make_out_map(&op->tmC, C, M, Cout, ldc, epi.flags)) return DLM_ERR_CUDA;
  p.M = M;
  p.N = Cout;
  p.num_kb = static_cast<int>(ktot / 64);
  p.m_tiles = pair ? (M + 2 * kGemmBM - 1) / (2 * kGemmBM) : M / kGemmBM;
  p.n_tiles = (Cout + bn - 1) / bn;
  p.stats_ld = p.n_tiles;
  p.amode = 1;
  p.oH = oH;
  p.oW = oW;
  p.bh = bh;
  p.bw = bw;
  p.nseg = nsrc;
  p.out = C;
  p.ldo = ldc;
  fill_epilogue(p, epi, p.N);
  p.status = device_status_ptr();
  op->bn = bn;
  op->pair = pair;
  op->k_true = ktot;
  set_grid(op, sk_bn != 0, epi);
  return DLM_OK;
}

int gemm_prepare_kernels() {
  // Sets the dynamic shared-memory limit of every tile variant up front, so that no attribute
  // call happens inside a CUDA-graph capture.
  int rc = gemm_prepare_fl<kEpiDyn>();
#define DLM_GEMM_PREPARE(F) \
  if (rc == DLM_OK) rc = gemm_prepare_fl<F>();
  DLM_GEMM_SPECIAL_FLAGS(DLM_GEMM_PREPARE)
#undef DLM_GEMM_PREPARE
  return rc;
}

int gemm_launch(const GemmOp& op, cudaStream_t s) {
  static bool prepared[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !prepared[dev]) {
    const int rc = gemm_prepare_kernels();
    if (rc != DLM_OK) return rc;
    prepared[dev] = true;
  }
  switch (op.p.flags) {
#define DLM_GEMM_CASE(F) \
  case F:                \
    return gemm_launch_fl<F>(op, s);
    DLM_GEMM_SPECIAL_FLAGS(DLM_GEMM_CASE)
#undef DLM_GEMM_CASE
    default:
      return gemm_launch_fl<kEpiDyn>(op, s);
  }
}

template int gemm_launch_fl<kEpiDyn>(const GemmOp&, cudaStream_t);
template int gemm_prepare_fl<kEpiDyn>();

}  // namespace dlm

extern "C" {

int dlm_gemm_set_tile_mode(int mode) {
  const int kernel = mode & 15, bn = mode >> 4;
  DLM_REQUIRE(kernel >= 0 && kernel <= 3, DLM_ERR_INVALID,
              "gemm_set_tile_mode: low bits 0 auto, 1 single, 2 pair, 3 stream-K");
  DLM_REQUIRE(bn == 0 || bn == 64 || bn == 128 || bn == 160 || bn == 192 || bn == 224 || bn == 256,
              DLM_ERR_INVALID, "gemm_set_tile_mode: forced tile width %d", bn);
  dlm::g_force_mode = kernel;
  dlm::g_force_bn = bn;
  return DLM_OK;
}

int dlm_gemm_fp16_ex(const void* A, int lda, const void* W, void* C, int ldc, int M, int N, int K,
                     unsigned flags, const void* bias, const void* bias2d, int rows_per_img,
                     const void* residual, int ldr, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  dlm::GemmEpilogue e;
  e.flags = flags;
  e.bias = static_cast<const __half*>(bias);
  e.bias2d = static_cast<const __half*>(bias2d);
  e.rows_per_img = rows_per_img;
  e.resid = static_cast<const __half*>(residual);
  e.ldr = ldr;
  dlm::GemmOp op;
  int rc = dlm::gemm_plan_dense(&op, static_cast<const __half*>(A), lda,
                                static_cast<const __half*>(W), M, N, K, static_cast<__half*>(C),
                                ldc, e);
  if (rc != DLM_OK) return rc;
  return dlm::gemm_launch(op, static_cast<cudaStream_t>(stream));
}

size_t dlm_gemm_workspace_bytes(void) { return dlm::gemm_sk_workspace_bytes(); }

int dlm_gemm_fp16_ws(const void* A, int lda, const void* W, void* C, int ldc, int M, int N, int K,
                     unsigned flags, const void* bias, const void* residual, int ldr, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  DLM_REQUIRE(workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
              DLM_ERR_INVALID, "gemm_fp16_ws: workspace must be 256-byte aligned");
  DLM_REQUIRE(!(flags & ~(DLM_EPI_BIAS | DLM_EPI_RESID | DLM_EPI_GEGLU | DLM_EPI_SILU)),
              DLM_ERR_INVALID, "gemm_fp16_ws: flags");
  dlm::GemmEpilogue e;
  e.flags = flags;
  e.bias = static_cast<const __half*>(bias);
  e.resid = static_cast<const __half*>(residual);
  e.ldr = ldr;
  e.sk_ws = workspace;
  e.sk_ws_bytes = workspace ? workspace_bytes : 0;
  dlm::GemmOp op;
  int rc = dlm::gemm_plan_dense(&op, static_cast<const __half*>(A), lda,
                                static_cast<const __half*>(W), M, N, K, static_cast<__half*>(C),
                                ldc, e);
  if (rc != DLM_OK) return rc;
  return dlm::gemm_launch(op, static_cast<cudaStream_t>(stream));
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Any shape and orientation: the operands are gathered (transposed where needed) into
// zero-padded [M, Kp] / [Np, Kp] stream-ordered scratch (Kp = K rounded up to 8, Np = N rounded
// up to 32), the product goes to [M, Np] scratch (seeded from C when beta != 0) and its first N
// columns are copied back.
int gemm_fp16_padded(const __half* A, const __half* B, __half* C, int M, int N, int K, float alpha,
                     float beta, int transA, int transB, cudaStream_t s) {
  const int Kp = (K + 7) / 8 * 8, Np = (N + 31) / 32 * 32;
  const size_t na = static_cast<size_t>(M) * Kp, nb = static_cast<size_t>(Np) * Kp,
               nc = static_cast<size_t>(M) * Np;
  __half* buf = nullptr;
  DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&buf), (na + nb + nc) * 2 + 512, s));
  __half* a = buf;
  __half* b = a + (na + 127) / 128 * 128;
  __half* c = b + (nb + 127) / 128 * 128;
  int rc = dlm::gather_pad(A, transA ? 1 : K, transA ? M : 1, M, K, a, M, Kp, s);
  if (rc == DLM_OK) rc = dlm::gather_pad(B, transB ? K : 1, transB ? 1 : N, N, K, b, Np, Kp, s);
  dlm::GemmEpilogue e;
  e.alpha = alpha;
  if (rc == DLM_OK && beta != 0.0f) {
    rc = dlm::gather_pad(C, N, 1, M, N, c, M, Np, s);
    e.flags |= DLM_EPI_RESID;
    e.resid = c;
    e.ldr = Np;
    e.resid_scale = beta;
  }
  dlm::GemmOp op;
  if (rc == DLM_OK) rc = dlm::gemm_plan_dense(&op, a, Kp, b, M, Np, Kp, c, Np, e);
  if (rc == DLM_OK) rc = dlm::gemm_launch(op, s);
  if (rc == DLM_OK) rc = dlm::gather_pad(c, Np, 1, M, N, C, M, N, s);
  cudaFreeAsync(buf, s);
  return rc;
}

}  // namespace

int dlm_launch_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                         float beta, int transA, int transB, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  DLM_REQUIRE(A && B && C, DLM_ERR_INVALID, "dlm_launch_gemm_fp16: null pointer");
  DLM_REQUIRE(M > 0 && N > 0 && K > 0, DLM_ERR_INVALID, "dlm_launch_gemm_fp16: negative size");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K % 8 != 0 || N % 32 != 0 || !aligned16(A) || !aligned16(B) || !aligned16(C) ||
      (transA && M % 8 != 0) || (!transB && N % 8 != 0))
    return gemm_fp16_padded(static_cast<const __half*>(A), static_cast<const __half*>(B),
                            static_cast<__half*>(C), M, N, K, alpha, beta, transA, transB, s);
  // The tensor-core kernel reads A as [M, K] and B as [N, K] (both K-major); the other
  // orientations are transposed once into stream-ordered scratch.
  __half* at = nullptr;
  __half* bt = nullptr;
  const __half* a = static_cast<const __half*>(A);
  const __half* b = static_cast<const __half*>(B);
  if (transA) {
    DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&at), static_cast<size_t>(M) * K * 2, s));
    int rc = dlm::transpose_strided(a, M, at, K, M, s);  // [K, M] -> [M, K]
    if (rc != DLM_OK) {
      cudaFreeAsync(at, s);
      return rc;
    }
    a = at;
  }
  if (!transB) {
    DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&bt), static_cast<size_t>(N) * K * 2, s));
    int rc = dlm::transpose_strided(b, N, bt, K, N, s);  // [K, N] -> [N, K]
    if (rc != DLM_OK) {
      if (at) cudaFreeAsync(at, s);
      cudaFreeAsync(bt, s);
      return rc;
    }
    b = bt;
  }
  dlm::GemmEpilogue e;
  e.alpha = alpha;
  if (beta != 0.0f) {
    e.flags |= DLM_EPI_RESID;
    e.resid = static_cast<const __half*>(C);
    e.ldr = N;
    e.resid_scale = beta;
  }
  dlm::GemmOp op;
  int rc = dlm::gemm_plan_dense(&op, a, K, b, M, N, K, static_cast<__half*>(C), N, e);
  if (rc == DLM_OK) rc = dlm::gemm_launch(op, s);
  if (at) cudaFreeAsync(at, s);
  if (bt) cudaFreeAsync(bt, s);
  return rc;
}

int dlm_gemm_fp16_batched(const void* A, const void* B, void* C, int batch, int M, int N, int K,
                          long long stride_a, long long stride_b, long long stride_c, float alpha,
                          float beta, int trans_b, void* stream) {
  if (batch <= 0 || M == 0 || N == 0 || K == 0) return DLM_OK;
  DLM_REQUIRE(A && B && C && M > 0 && N > 0 && K > 0 && stride_a >= 0 && stride_b >= 0 && stride_c >= 0,
              DLM_ERR_INVALID, "dlm_gemm_fp16_batched: bad descriptor");
  for (int i = 0; i < batch; ++i) {
    const int rc = dlm_launch_gemm_fp16(static_cast<const __half*>(A) + i * stride_a,
                                        static_cast<const __half*>(B) + i * stride_b,
                                        static_cast<__half*>(C) + i * stride_c, M, N, K, alpha, beta, 0,
                                        trans_b, stream);
    if (rc != DLM_OK) return rc;
  }
  return DLM_OK;
}

}  // extern "C"
