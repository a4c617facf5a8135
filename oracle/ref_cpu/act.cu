// cpu_silu / cpu_gelu_erf / cpu_gelu_tanh of src/tests/test_activation.cu (act 0 / 1 / 2).
#define main dollama_ref_test_main
#include "tests/test_activation.cu"
#undef main
extern "C" int ref_cpu_activation(const float* in, size_t n, int act, float* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = act == 0 ? dollama::cpu_silu(in[i]) : act == 1 ? dollama::cpu_gelu_erf(in[i]) : dollama::cpu_gelu_tanh(in[i]);
  return 0;
}
