// cpu_group_norm of src/tests/test_groupnorm.cu (one-pass fp32 sum / sum of squares).
#define main dollama_ref_test_main
#include "tests/test_groupnorm.cu"
#undef main
extern "C" int ref_cpu_group_norm(const float* in, const float* gamma, const float* beta, int N, int C,
                                  int H, int W, int G, float eps, float* out) {
  std::vector<float> x(in, in + static_cast<size_t>(N) * C * H * W), g(gamma, gamma + C), b(beta, beta + C);
  const std::vector<float> r = dollama::cpu_group_norm(x, g, b, N, C, H, W, G, eps);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
