// BitNet ternary tag LM model object (bitnet_lm.cu).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "common.h"

namespace dlm {

struct BitNetCfg {
  int vocab = 16000, d_model = 512, n_layers = 8, n_heads = 8, ffn_dim = 1536, max_seq = 128;
  double rope_base = 10000.0, rms_eps = 1e-5;
  int per_tensor_scale = 0;
};

struct BitNetWeightSpec {
  std::string name;
  std::vector<int64_t> shape;
};
std::vector<BitNetWeightSpec> bitnet_weight_specs(const BitNetCfg& c);
int bitnet_check_cfg(const BitNetCfg& c);

class BitNetLM {
 public:
  ~BitNetLM();
  int create(const BitNetCfg& cfg, int n, const char* const* names, const float* const* ptrs,
             const int64_t* numels, cudaStream_t s);
  // logits [B, S, vocab] of every position of tokens [B, S] (host or device pointers).
  int forward(const int* tokens, int B, int S, float* logits, cudaStream_t s);
  // Greedy decode of prompts [B, P] up to max_len tokens per sequence: out [B, max_len - P]
  // generated ids, out_len [B] their counts (host or device pointers).  Returns when done.
  int generate(const int* prompts, int B, int P, int max_len, int* out, int* out_len, cudaStream_t s);
  size_t arena_bytes() const { return arena_bytes_; }

 private:
  struct Layer {
    float *attn_norm = nullptr, *ffn_norm = nullptr;
    uint32_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;  // 2-bit packed
    float *aqkv = nullptr, *ao = nullptr, *agu = nullptr, *ad = nullptr;     // row scales
  };
  template <typename T>
  T* walloc(size_t n);
  int plan(int B, int P, int Lmax, bool all_logits);
  void release_plan();
  int set_smem_attrs();
  int run_layers(int S, const int* pos, cudaStream_t s);
  int run_head(int rows, int stride, int off, cudaStream_t s);
  int decode_step(cudaStream_t s);
  int check_bad(cudaStream_t s);

  BitNetCfg cfg_;
  std::vector<void*> wallocs_;
  float *embed_ = nullptr, *final_norm_ = nullptr;
  double* embT_ = nullptr;  // the embedding transposed, [d_model][ldv_], double (lm_head operand)
  int ldv_ = 0;
  double *cos_t_ = nullptr, *sin_t_ = nullptr;
  std::vector<Layer> layers_;
  // plan
  int B_ = 0, P_ = 0, L_ = 0;
  bool all_logits_ = false;
  void* abuf_ = nullptr;
  size_t arena_bytes_ = 0;
  int* tokens_ = nullptr;
  float *h_ = nullptr, *xs_ = nullptr, *y_ = nullptr, *q_ = nullptr, *ao_ = nullptr;
  int8_t* xq_ = nullptr;
  float *kc_ = nullptr, *vc_ = nullptr, *logits_ = nullptr;
  double* normT_ = nullptr;  // the final norm's rows transposed, [d_model][ldx_], double
  int ldx_ = 0;
  int *state_ = nullptr, *done_ = nullptr, *out_ = nullptr, *out_len_ = nullptr;
  cudaGraphExec_t step_graph_ = nullptr;
  cudaStream_t cap_stream_ = nullptr;
};

}  // namespace dlm
