// C entry points onto the reference's OWN BitNet integer path — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_oracle.py (when the reference tree is present) from the reference's
// header src/models/bitnet.hpp where it lies, into oracle/_ref/libref_bitnet.so.  It lets the
// tests pin the C restatement (bitnet_oracle.c) and the GPU kernels against the reference's own
// quantize_weight_ternary / quantize_activation_int8 (bitnet.hpp:70-165) and BitNet::bitlinear
// (bitnet.hpp:447-471, a private static member, reached by opening the class's access here).
#include <cstddef>
#include <cstdint>
#include <cstring>

#define private public
#include "models/bitnet.hpp"
#undef private

extern "C" {

float ref_quantize_weight_ternary(const float* w, size_t n, int8_t* q) {
  const dollama::TernaryQuant r = dollama::quantize_weight_ternary(w, n);
  if (n) std::memcpy(q, r.q.data(), n);
  return r.scale;
}

float ref_quantize_activation_int8(const float* x, size_t n, int8_t* q) {
  const dollama::Int8Quant r = dollama::quantize_activation_int8(x, n);
  if (n) std::memcpy(q, r.q.data(), n);
  return r.scale;
}

void ref_bitlinear(const float* w, const float* x, int out_dim, int in_dim, float* y) {
  dollama::BitNet::bitlinear(w, x, out_dim, in_dim, y);
}

}  // extern "C"
