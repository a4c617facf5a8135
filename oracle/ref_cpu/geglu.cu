// cpu_geglu of src/tests/test_geglu.cu: [tokens, 2d] -> x1 * gelu_erf(x2).
#define main dollama_ref_test_main
#include "tests/test_geglu.cu"
#undef main
extern "C" int ref_cpu_geglu(const float* in, int tokens, int d, float* out) {
  std::vector<float> x(in, in + static_cast<size_t>(tokens) * 2 * d);
  const std::vector<float> r = dollama::cpu_geglu(x, tokens, d);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
