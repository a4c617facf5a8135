// SDXL UNet model object: prepared weights, static activation arena, op plan, CUDA graph.
#pragma once

#include <functional>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_fp16.h>

#include "attention.h"
#include "common.h"
#include "gemm.h"
#include "norm.h"
#include "plan.h"

namespace dlm {

struct UNetCfg {
  int depth[3] = {0, 2, 10};  // transformer layers per Transformer2D at 1x, 1/2x, 1/4x
  int mid_depth = 10;
};

struct ResnetInfo {
  std::string prefix;
  int cin, cout;
  int temb_off;  // column offset of this resnet in the concatenated time-embedding projection
};

// Where a diffusers weight [out, in_flat] lives in the prepared weights (runtime LoRA / restore).
struct LoraTarget {
  __half* w = nullptr;  // prepared matrix
  int ld = 0;           // its row stride (elements)
  int row_off = 0, col_off = 0;
  int kind = 0;         // 0 rows / columns as given, 1 conv [o][i][tap] -> [o][tap][i], 2 GEGLU rows
  int kk = 1, cin = 0, cin_pad = 0;
  int half_rows = 0;    // GEGLU: rows per half (row r < half -> 2r, else 2(r - half) + 1)
  // LayerNorm fold (gamma != nullptr): the folded matrix has in_flat columns
  const __half* gamma = nullptr;
  const __half* beta = nullptr;
  const __half* bias = nullptr;  // bias term of v per prepared row
  float* u = nullptr;
  float* v = nullptr;
};

class UNetModel {
 public:
  ~UNetModel();
  int create(const UNetCfg& cfg, int n, const char* const* names, const void* const* ptrs,
             const int64_t* numels, cudaStream_t s);
  int forward(int B, int H, int W, const __half* latent, float timestep, const __half* ehs,
              const __half* te, const __half* tid, __half* noise_out, cudaStream_t s);
  // Same step with pinned/pageable HOST inputs and output; returns after the result is on host.
  int forward_host(int B, int H, int W, const __half* latent, float timestep, const __half* ehs,
                   const __half* te, const __half* tid, __half* noise_out, cudaStream_t s);
  static constexpr int kNumOpClasses = OpPlan::kNumClasses;
  int time_ops(cudaStream_t s, double* ms, double* flops, int* count);
  void set_graph(bool on) {
    if (on != use_graph_) ops_.drop_graph();
    use_graph_ = on;
  }
  int stage(const std::string& name, const __half** ptr, int* C, int* H, int* W) const;
  // Runtime LoRA: W += scale * (B A) merged into the prepared (packed / folded) copy of the
  // diffusers weight `key` (A [rank, in_flat], B [out, rank], fp16 device).  The prepared rows it
  // touches are saved first; clear_loras writes every saved block back, newest first, so the
  // weights return bit for bit to their state before the first apply.
  int apply_lora(const std::string& key, const __half* A, const __half* B, int rank, int in_flat,
                 int out, float scale, cudaStream_t s);
  int clear_loras(cudaStream_t s);
  int num_lora_patches() const { return static_cast<int>(patches_.size()); }
  size_t arena_bytes() const { return arena_bytes_; }
  size_t weight_bytes() const { return woff_; }
  int num_launches() const { return ops_.num_launches(); }

 private:
  struct StageInfo {
    const __half* ptr;
    int C, H, W;
  };

  int prepare_weights(cudaStream_t s);
  int lora_target(const std::string& key, struct LoraTarget* t, int* out, int* in_flat) const;
  // one saved block of prepared rows (and their LayerNorm-fold sums) per apply_lora
  struct LoraPatch {
    __half* w;       // first saved row of the prepared matrix
    size_t elems;    // rows * ld
    float* u;        // fold sums of those rows (nullptr when unfolded)
    float* v;
    int rows;
    void* saved;     // device copy: elems halves, then 2 * rows floats
  };
  const __half* src(const std::string& n) const;
  const __half* W(const std::string& n) const;
  const float* WF(const std::string& n) const;
  __half* wtake(size_t elems);
  __half* act(size_t elems);
  int plan(int B, int H, int W);
  int build(bool dry);
  void release_plan();
  int launch_step(float timestep, cudaStream_t s);
  int plan_gn(const __half* x1, int C1, const __half* x2, int C2, int HW, const std::string& wprefix,
              float eps, bool silu, __half* out);
  int plan_resnet(const ResnetInfo& rs, const __half* x1, int C1, const __half* x2, int C2, int H,
                  int W, __half* out);
  int plan_t2d(const std::string& p, __half* x, int C, int H, int W, int layers);
  int plan_linear(const __half* A, int lda, const __half* Wt, int M, int N, int K, __half* C, int ldc,
                  const GemmEpilogue& e, int* bn_out = nullptr);
  int plan_attn(const __half* q, int ldq, const __half* k, int ldk, const __half* v, int ldv,
                __half* o, int ldo, int heads, int Sq, int Sk);
  void push_gemm(const GemmOp& g, double flops = -1.0) { ops_.push_gemm(g, flops); }
  void push_attn(const AttnOp& a) { ops_.push_attn(a); }
  void push_gn(const GnOp& g) { ops_.push_gn(g); }
  void push_ln(const LnArgs& l) { ops_.push_ln(l); }
  void push_custom(std::function<int(cudaStream_t)> f) { ops_.push_custom(std::move(f)); }

  UNetCfg cfg_;
  // weights
  std::unordered_map<std::string, const __half*> src_;  // caller's tensors (create only)
  std::unordered_map<std::string, __half*> w_;          // prepared tensors
  std::unordered_map<std::string, float*> wf_;          // prepared fp32 vectors (LN fold u / v)
  void* wbuf_ = nullptr;
  size_t wcap_ = 0, woff_ = 0;
  std::vector<ResnetInfo> resnets_;
  __half* kv_all_w_ = nullptr;                          // [kv_total_, 2048] all cross k/v weights
  int kv_total_ = 0, kv_cursor_ = 0;
  std::unordered_map<std::string, int> kv_off_;         // block prefix -> row offset in kv_all_w_
  std::vector<LoraPatch> patches_;                      // applied LoRAs, oldest first
  int temb_total_ = 0;
  // plan
  int B_ = 0, H_ = 0, W_ = 0;
  bool dry_ = false;
  void* abuf_ = nullptr;
  size_t arena_bytes_ = 0;
  ActArena arena_;
  OpPlan ops_;
  std::unordered_map<std::string, StageInfo> stages_;
  bool use_graph_ = true;
  // buffers inside the arena
  float* d_t_ = nullptr;
  __half *tid_ = nullptr, *te_ = nullptr, *ehs_ = nullptr, *lat_in_ = nullptr, *noise_out_ = nullptr;
  __half *lat64_ = nullptr, *tproj_ = nullptr;
  __half *scratch_a_ = nullptr, *scratch_b_ = nullptr, *scratch_c_ = nullptr;
  __half *t_gn_ = nullptr, *t_h_ = nullptr, *t_n_ = nullptr, *t_qkv_ = nullptr, *t_ao_ = nullptr,
         *t_ff_ = nullptr, *kv_all_act_ = nullptr;
  __half *planes_ = nullptr, *upbuf_ = nullptr, *out32_ = nullptr;
  float2* gn_partials_ = nullptr;
  float2* ln_stats_ = nullptr;
  size_t gn_partial_cap_ = 0;
  void* attn_ws_ = nullptr;  // stream-K attention workspace shared by every attention launch
  size_t attn_ws_bytes_ = 0;
};

}  // namespace dlm
