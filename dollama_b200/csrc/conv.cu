// C-ABI entry points of the implicit-GEMM convolution and its layout helpers.
#include "gemm.h"
#include "ops.h"

extern "C" {

size_t dlm_conv2d_nhwc_scratch_bytes(int N, int H, int W, int Cin, int ksize, int stride) {
  if (ksize == 3 && stride == 2) return static_cast<size_t>(N) * H * W * Cin * sizeof(__half);
  return 0;
}

int dlm_conv2d_nhwc(const void* in, int N, int H, int W, int Cin, const void* w_krsc,
                    const void* bias, void* out, int Cout, int ksize, int stride, void* scratch,
                    size_t scratch_bytes, void* stream) {
  if (N == 0 || H == 0 || W == 0 || Cin == 0 || Cout == 0) return DLM_OK;
  DLM_REQUIRE(in && w_krsc && out, DLM_ERR_INVALID, "conv2d_nhwc: null pointer");
  DLM_REQUIRE((ksize == 3 && (stride == 1 || stride == 2)) || (ksize == 1 && stride == 1),
              DLM_ERR_UNSUPPORTED, "conv2d_nhwc: only 3x3 (stride 1/2, pad 1) and 1x1 supported");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dlm::GemmEpilogue e;
  if (bias) {
    e.flags |= DLM_EPI_BIAS;
    e.bias = static_cast<const __half*>(bias);
  }
  dlm::ConvSource src;
  src.C = Cin;
  int oH = H, oW = W;
  if (stride == 2) {
    DLM_REQUIRE(H % 2 == 0 && W % 2 == 0, DLM_ERR_INVALID, "conv2d_nhwc: stride 2 needs even H, W");
    const size_t need = dlm_conv2d_nhwc_scratch_bytes(N, H, W, Cin, ksize, stride);
    DLM_REQUIRE(scratch != nullptr && scratch_bytes >= need, DLM_ERR_INVALID,
                "conv2d_nhwc: stride 2 needs %zu scratch bytes", need);
    DLM_REQUIRE(Cin % 8 == 0, DLM_ERR_INVALID, "conv2d_nhwc: Cin %% 8");
    oH = H / 2;
    oW = W / 2;
    int rc = dlm::parity_planes(static_cast<const __half*>(in), static_cast<__half*>(scratch), N, H,
                                W, Cin, s);
    if (rc != DLM_OK) return rc;
    src.kind = 2;
    src.ptr = static_cast<const __half*>(scratch);
  } else {
    src.kind = ksize == 3 ? 0 : 1;
    src.ptr = static_cast<const __half*>(in);
  }
  dlm::GemmOp op;
  int rc = dlm::gemm_plan_conv(&op, N, oH, oW, &src, 1, static_cast<const __half*>(w_krsc), Cout,
                               static_cast<__half*>(out), Cout, e);
  if (rc != DLM_OK) return rc;
  return dlm::gemm_launch(op, s);
}

int dlm_pack_conv_weight(const void* w_oihw, void* w_krsc, int Cout, int Cin, int KH, int KW,
                         void* stream) {
  if (Cout == 0 || Cin == 0 || KH == 0 || KW == 0) return DLM_OK;
  DLM_REQUIRE(w_oihw && w_krsc, DLM_ERR_INVALID, "pack_conv_weight: null pointer");
  return dlm::pack_conv_weight(static_cast<const __half*>(w_oihw), static_cast<__half*>(w_krsc),
                               Cout, Cin, KH, KW, static_cast<cudaStream_t>(stream));
}

int dlm_nchw_to_nhwc(const void* in, void* out, int N, int C, int HW, void* stream) {
  if (N == 0 || C == 0 || HW == 0) return DLM_OK;
  DLM_REQUIRE(in && out && in != out, DLM_ERR_INVALID, "nchw_to_nhwc: bad pointers");
  return dlm::nchw_to_nhwc(static_cast<const __half*>(in), static_cast<__half*>(out), N, C, HW,
                           static_cast<cudaStream_t>(stream));
}

int dlm_nhwc_to_nchw(const void* in, void* out, int N, int C, int HW, void* stream) {
  if (N == 0 || C == 0 || HW == 0) return DLM_OK;
  DLM_REQUIRE(in && out && in != out, DLM_ERR_INVALID, "nhwc_to_nchw: bad pointers");
  return dlm::nhwc_to_nchw(static_cast<const __half*>(in), static_cast<__half*>(out), N, C, HW,
                           static_cast<cudaStream_t>(stream));
}

}  // extern "C"
