// cpu_layer_norm of src/tests/test_layernorm.cu.
#define main dollama_ref_test_main
#include "tests/test_layernorm.cu"
#undef main
extern "C" int ref_cpu_layer_norm(const float* in, const float* gamma, const float* beta, int rows, int C,
                                  float eps, float* out) {
  std::vector<float> x(in, in + static_cast<size_t>(rows) * C);
  std::vector<float> g = gamma ? std::vector<float>(gamma, gamma + C) : std::vector<float>();
  std::vector<float> b = beta ? std::vector<float>(beta, beta + C) : std::vector<float>();
  const std::vector<float> r = dollama::cpu_layer_norm(x, g, b, rows, C, eps);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
