// cpu_attention of src/tests/test_attention.cu: q [B, H, Sq, Dh], k / v [B, H, Sk, Dh].
#define main dollama_ref_test_main
#include "tests/test_attention.cu"
#undef main
extern "C" int ref_cpu_attention(const float* q, const float* k, const float* v, int B, int H, int Sq,
                                 int Sk, int Dh, float scale, float* out) {
  std::vector<float> vq(q, q + static_cast<size_t>(B) * H * Sq * Dh);
  std::vector<float> vk(k, k + static_cast<size_t>(B) * H * Sk * Dh);
  std::vector<float> vv(v, v + static_cast<size_t>(B) * H * Sk * Dh);
  const std::vector<float> r = dollama::cpu_attention(vq, vk, vv, B, H, Sq, Sk, Dh, scale);
  std::copy(r.begin(), r.end(), out);
  return 0;
}
