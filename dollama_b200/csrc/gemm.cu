// Host side of the tcgen05 GEMM: tile-width choice, tensor-map encoding, launch, and the
// GEMM entry points of the C ABI.
#include <cstring>

#include "gemm.h"

namespace dlm {

namespace {

template <int BN>
int launch_bn(const GemmOp& op, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        gemm_smem_bytes(BN)));
    attr_set[dev] = true;
  }
  gemm_tc_kernel<BN><<<op.grid, kGemmThreads, gemm_smem_bytes(BN), s>>>(op.tmA[0], op.tmA[1],
                                                                         op.tmA[2], op.tmB, op.p);
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

// Relative cost of one 128 x BN tile per unit of K: MMA time grows with BN; narrow tiles are
// bound by shared-memory operand bandwidth (A + B bytes per MMA); plus a fixed per-tile cost.
double tile_cost(int bn) {
  const double mma = bn;
  const double smem = 0.5 * (128 + bn);
  return (mma > smem ? mma : smem) + 24.0;
}

int pick_bn(int M, int N) {
  static const int cands[] = {256, 192, 160, 128, 64};
  const int sms = num_sms();
  const int m_tiles = (M + kGemmBM - 1) / kGemmBM;
  int best = 128;
  double best_cost = 1e30;
  for (int bn : cands) {
    const int n_tiles = (N + bn - 1) / bn;
    const long tiles = static_cast<long>(m_tiles) * n_tiles;
    const long waves = (tiles + sms - 1) / sms;
    const double cost = waves * tile_cost(bn);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

bool bn_supported(int bn) { return bn == 256 || bn == 192 || bn == 160 || bn == 128 || bn == 64; }

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
    DLM_REQUIRE(!(e.flags & DLM_EPI_RESID) && N % 64 == 0, DLM_ERR_INVALID,
                "gemm: GEGLU needs N %% 64 == 0 and no residual");
  return DLM_OK;
}

}  // namespace

int gemm_plan_dense(GemmOp* op, const __half* A, int lda, const __half* W, int M, int N, int K,
                    __half* C, int ldc, const GemmEpilogue& epi, int force_bn) {
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
  const int bn = force_bn ? force_bn : pick_bn(M, N);
  DLM_REQUIRE(bn_supported(bn), DLM_ERR_INVALID, "gemm: unsupported tile width %d", bn);
  std::memset(op, 0, sizeof(*op));
  if (!tmap_2d_f16(&op->tmA[0], A, M, K, lda, kGemmBM, kGemmBK)) return DLM_ERR_CUDA;
  op->tmA[1] = op->tmA[0];
  op->tmA[2] = op->tmA[0];
  if (!tmap_2d_f16(&op->tmB, W, N, K, K, bn, kGemmBK)) return DLM_ERR_CUDA;
  GemmParams& p = op->p;
  p.M = M;
  p.N = N;
  p.num_kb = (K + kGemmBK - 1) / kGemmBK;
  p.m_tiles = (M + kGemmBM - 1) / kGemmBM;
  p.n_tiles = (N + bn - 1) / bn;
  p.amode = 0;
  p.out = C;
  p.ldo = ldc;
  fill_epilogue(p, epi, p.N);
  p.status = device_status_ptr();
  op->bn = bn;
  op->k_true = K;
  const int tiles = p.m_tiles * p.n_tiles;
  op->grid = tiles < num_sms() ? tiles : num_sms();
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
  const int bn = force_bn ? force_bn : pick_bn(M, Cout);
  DLM_REQUIRE(bn_supported(bn), DLM_ERR_INVALID, "conv: unsupported tile width %d", bn);
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
  if (!tmap_2d_f16(&op->tmB, W, Cout, ktot, ktot, bn, kGemmBK)) return DLM_ERR_CUDA;
  p.M = M;
  p.N = Cout;
  p.num_kb = static_cast<int>(ktot / 64);
  p.m_tiles = M / kGemmBM;
  p.n_tiles = (Cout + bn - 1) / bn;
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
  op->k_true = ktot;
  const int tiles = p.m_tiles * p.n_tiles;
  op->grid = tiles < num_sms() ? tiles : num_sms();
  return DLM_OK;
}

int gemm_prepare_kernels() {
  // Sets the dynamic shared-memory limit of every tile variant up front, so that no attribute
  // call happens inside a CUDA-graph capture.
  GemmOp dummy;
  std::memset(&dummy, 0, sizeof(dummy));
  (void)dummy;
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(256)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<192>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(192)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<160>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(160)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(128)));
  DLM_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(64)));
  return DLM_OK;
}

int gemm_launch(const GemmOp& op, cudaStream_t s) {
  switch (op.bn) {
    case 256: return launch_bn<256>(op, s);
    case 192: return launch_bn<192>(op, s);
    case 160: return launch_bn<160>(op, s);
    case 128: return launch_bn<128>(op, s);
    case 64: return launch_bn<64>(op, s);
    default: set_error("gemm: op not planned"); return DLM_ERR_INVALID;
  }
}

}  // namespace dlm

extern "C" {

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

int dlm_launch_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                         float beta, int transA, int transB, void* stream) {
  if (M == 0 || N == 0 || K == 0) return DLM_OK;
  DLM_REQUIRE(!transA && transB, DLM_ERR_UNSUPPORTED,
              "dlm_launch_gemm_fp16: only transA=0, transB=1 is provided");
  dlm::GemmEpilogue e;
  e.alpha = alpha;
  if (beta != 0.0f) {
    e.flags |= DLM_EPI_RESID;
    e.resid = static_cast<const __half*>(C);
    e.ldr = N;
    e.resid_scale = beta;
  }
  dlm::GemmOp op;
  int rc = dlm::gemm_plan_dense(&op, static_cast<const __half*>(A), K,
                                static_cast<const __half*>(B), M, N, K, static_cast<__half*>(C), N,
                                e);
  if (rc != DLM_OK) return rc;
  return dlm::gemm_launch(op, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
