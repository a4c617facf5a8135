// cpu_time_embedding of src/tests/test_timeembed.cu ([cos | sin], max_period).
#define main dollama_ref_test_main
#include "tests/test_timeembed.cu"
#undef main
extern "C" int ref_cpu_time_embedding(float t, int dim, float max_period, float* out) {
  const std::vector<float> r = dollama::cpu_time_embedding(t, dim, max_period);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
