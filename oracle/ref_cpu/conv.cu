// cpu_conv2d of src/tests/test_conv2d.cu (direct NCHW convolution, fp32).  The test's GPU entry
// points are left unresolved (its kernels link cuBLAS): the library is opened with lazy binding
// and only this CPU function is ever called.
#define main dollama_ref_test_main
#include "tests/test_conv2d.cu"
#undef main
extern "C" int ref_cpu_conv2d(const float* in, const float* w, const float* bias, int N, int Cin, int H,
                              int W, int Cout, int KH, int KW, int stride, int pad, float* out) {
  std::vector<float> x(in, in + static_cast<size_t>(N) * Cin * H * W);
  std::vector<float> wt(w, w + static_cast<size_t>(Cout) * Cin * KH * KW);
  std::vector<float> b = bias ? std::vector<float>(bias, bias + Cout) : std::vector<float>();
  const std::vector<float> r =
      dollama::cpu_conv2d(x, wt, b, N, Cin, H, W, Cout, KH, KW, stride, stride, pad, pad, 1, 1);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
