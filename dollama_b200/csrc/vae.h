// SDXL AutoencoderKL decoder: prepared weights, static activation arena, op plan, CUDA graph.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_fp16.h>

#include "common.h"
#include "plan.h"

namespace dlm {

struct VaeWeightSpec {
  std::string name;
  std::vector<int64_t> shape;
};
std::vector<VaeWeightSpec> vae_weight_specs();

class VAEModel {
 public:
  ~VAEModel();
  int create(int n, const char* const* names, const void* const* ptrs, const int64_t* numels,
             cudaStream_t s);
  // latent [B, 4, h, w] fp16 (already divided by the scaling factor) -> image [B, 3, 8h, 8w] fp16.
  int decode(int B, int h, int w, const __half* latent, __half* image, cudaStream_t s);
  // Same with HOST latent / image (copies inside); returns after the image is on the host.
  int decode_host(int B, int h, int w, const __half* latent, __half* image, cudaStream_t s);
  int time_ops(cudaStream_t s, double* ms, double* flops, int* count);
  void set_graph(bool on) {
    if (on != use_graph_) ops_.drop_graph();
    use_graph_ = on;
  }
  // Named intermediate (NHWC), valid after a decode until the next one: dtype 0 fp16, 1 fp32.
  int stage(const std::string& name, const void** ptr, int* dtype, int* C, int* H, int* W) const;
  size_t arena_bytes() const { return arena_bytes_; }
  size_t weight_bytes() const { return woff_; }
  int num_launches() const { return ops_.num_launches(); }

 private:
  struct Act {  // an NHWC activation in the arena
    void* p = nullptr;
    bool f32 = false;
    int C = 0;
  };
  struct StageInfo {
    const void* ptr;
    int dtype, C, H, W;
  };

  int prepare_weights(cudaStream_t s);
  const __half* src(const std::string& n) const;
  const __half* W(const std::string& n) const;
  __half* wtake(size_t elems);
  int plan(int B, int h, int w);
  int build(bool dry);
  void release_plan();
  int plan_gn(const Act& x, int HW, const std::string& wprefix, bool silu, __half* out);
  int plan_resnet(const std::string& p, const Act& x, int cout, int H, int W, const Act& out);
  int plan_attn(const std::string& p, const Act& x, int H, int W);
  int plan_upsample(const std::string& p, const Act& x, int H, int W, const Act& out);

  std::unordered_map<std::string, const __half*> src_;  // caller's tensors (create only)
  std::unordered_map<std::string, __half*> w_;          // prepared tensors
  void* wbuf_ = nullptr;
  size_t wcap_ = 0, woff_ = 0;
  // plan
  int B_ = 0, h_ = 0, w_lat_ = 0;
  bool dry_ = false;
  void* abuf_ = nullptr;
  size_t arena_bytes_ = 0;
  ActArena arena_;
  OpPlan ops_;
  bool use_graph_ = true;
  std::unordered_map<std::string, StageInfo> stages_;
  // buffers inside the arena
  __half *lat_in_ = nullptr, *image_ = nullptr, *lat64_ = nullptr, *pqc_ = nullptr;
  __half *s_gn1_ = nullptr, *s_gn2_ = nullptr, *upbuf_ = nullptr, *out32_ = nullptr;
  void* s_c1_ = nullptr;  // conv1 output (fp16 or fp32)
  __half *qkv_ = nullptr, *attn_o_ = nullptr;
  float2* gn_partials_ = nullptr;
  size_t gn_partial_cap_ = 0;
};

}  // namespace dlm
