// A model step as a flat list of pre-encoded launches (GEMM / attention / GroupNorm / LayerNorm /
// custom), replayed eagerly or as one CUDA graph, plus the static activation arena the launches
// point into.  Shared by the UNet and VAE graphs: both plan once per input shape (a dry pass that
// only sizes the arena, then the real pass that encodes every tensor map), so a step allocates
// nothing and synchronises nothing on the host.
#pragma once

#include <functional>
#include <vector>

#include <cuda_fp16.h>

#include "attention.h"
#include "common.h"
#include "gemm.h"
#include "norm.h"

namespace dlm {

struct LnArgs {
  const __half* x;
  const __half* g;
  const __half* b;
  __half* out;
  int rows, C;
  float eps;
};

// Bump allocator over one device buffer.  In the dry pass it hands out fake (non-null,
// 256-byte aligned) addresses and only records the size the real pass will need.
class ActArena {
 public:
  void begin(bool dry, void* base) {
    dry_ = dry;
    base_ = base;
    off_ = 0;
  }
  template <typename T>
  T* take(size_t elems) {
    const size_t bytes = ((elems * sizeof(T) + 255) / 256) * 256;
    const size_t off = off_;
    off_ += bytes;
    if (dry_) return reinterpret_cast<T*>(static_cast<uintptr_t>(0x100000000ull + off));
    return reinterpret_cast<T*>(static_cast<char*>(base_) + off);
  }
  size_t used() const { return off_; }
  bool dry() const { return dry_; }

 private:
  bool dry_ = true;
  void* base_ = nullptr;
  size_t off_ = 0;
};

class OpPlan {
 public:
  static constexpr int kNumClasses = 5;  // gemm, attention, groupnorm, layernorm, other
  ~OpPlan();
  void clear();  // drops every op and the instantiated graph
  void push_gemm(const GemmOp& g, double flops = -1.0);
  void push_attn(const AttnOp& a);
  void push_attn_wide(const AttnWideOp& a);
  void push_gn(const GnOp& g);
  void push_ln(const LnArgs& l);
  void push_custom(std::function<int(cudaStream_t)> f, double flops = 0.0);
  // Eager launch of every op in order.
  int run(cudaStream_t s);
  // The step as one CUDA graph (captured on first use), or eager when `graph` is false.
  int replay(cudaStream_t s, bool graph);
  void drop_graph();
  // Per op class: device ms of the class's launches replayed alone as one CUDA graph (so the
  // classes add up to about the step graph's time), algorithmic FLOPs and launches.
  // DLM_OP_TABLE=<path> also writes one CSV line per launch of an eager, event-timed step.
  int time(cudaStream_t s, double* ms, double* flops, int* count);
  int num_launches() const;
  size_t size() const { return seq_.size(); }

 private:
  enum class Kind { Gemm, Attn, AttnWide, Gn, Ln, Custom };
  struct Ref {
    Kind kind;
    int idx;
  };
  int launch(const Ref& r, cudaStream_t s);
  int op_class(const Ref& r, double* flops) const;
  int write_table(cudaStream_t s, const char* path);
  std::vector<Ref> seq_;
  std::vector<GemmOp> gemm_;
  std::vector<double> gemm_flops_;
  std::vector<AttnOp> attn_;
  std::vector<AttnWideOp> attn_wide_;
  std::vector<GnOp> gn_;
  std::vector<LnArgs> ln_;
  std::vector<std::function<int(cudaStream_t)>> custom_;
  std::vector<double> custom_flops_;
  cudaGraphExec_t gexec_ = nullptr;
  cudaStream_t cap_stream_ = nullptr;
};

}  // namespace dlm
