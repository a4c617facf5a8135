// C entry points onto the reference's OWN BitNet integer path — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_oracle.py (when the reference tree is present) from the reference's
// header src/models/bitnet.hpp where it lies, into oracle/_ref/libref_bitnet.so.  It lets the
// tests pin the C restatement (bitnet_oracle.c) and the GPU kernels against the reference's own
// quantize_weight_ternary / quantize_activation_int8 (bitnet.hpp:70-165) and BitNet::bitlinear
// (bitnet.hpp:447-471, a private static member, reached by opening the class's access here), and
// the whole reference forward BitNet::forward (bitnet.hpp:376-440) at the reference's compiled-in
// dimensions (src/models/bitnet_config.hpp), with the weights set through the class's members.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

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

// dims[0..5] = vocab, d_model, n_layers, n_heads, ffn_dim, max_seq of the compiled reference.
void ref_bitnet_dims(int* dims) {
  dims[0] = dollama::BitNet::VOCAB_SIZE;
  dims[1] = dollama::BitNet::D_MODEL;
  dims[2] = dollama::BitNet::N_LAYERS;
  dims[3] = dollama::BitNet::N_HEADS;
  dims[4] = dollama::BitNet::FFN_DIM;
  dims[5] = dollama::BitNet::MAX_SEQ_LEN;
}

// logits [S, vocab] = BitNet::forward(tokens).  layer_w holds, per layer, the pointers
// attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up, w_down (9 per layer).  Returns 0, or -1
// when the reference throws (empty / too long sequence, token out of range).
int ref_bitnet_forward(const float* embed, const float* final_norm, const float* const* layer_w,
                       const int* tokens, int S, float* logits) {
  using dollama::BitNet;
  BitNet net;
  const size_t D = BitNet::D_MODEL, F = BitNet::FFN_DIM;
  net.embed_.assign(embed, embed + static_cast<size_t>(BitNet::VOCAB_SIZE) * D);
  net.final_norm_.assign(final_norm, final_norm + D);
  for (int l = 0; l < BitNet::N_LAYERS; ++l) {
    BitNet::Layer& L = net.layers_[l];
    const float* const* p = layer_w + 9 * l;
    L.attn_norm.assign(p[0], p[0] + D);
    L.wq.assign(p[1], p[1] + D * D);
    L.wk.assign(p[2], p[2] + D * D);
    L.wv.assign(p[3], p[3] + D * D);
    L.wo.assign(p[4], p[4] + D * D);
    L.ffn_norm.assign(p[5], p[5] + D);
    L.w_gate.assign(p[6], p[6] + F * D);
    L.w_up.assign(p[7], p[7] + F * D);
    L.w_down.assign(p[8], p[8] + D * F);
  }
  try {
    const std::vector<float> out = net.forward(std::vector<int>(tokens, tokens + S));
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
  } catch (...) {
    return -1;
  }
  return 0;
}

}  // extern "C"
