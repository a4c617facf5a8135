// OpPlan: eager / CUDA-graph replay and per-launch timing of a planned model step.
#include <cstdio>
#include <cstdlib>

#include "plan.h"

namespace dlm {

OpPlan::~OpPlan() { clear(); }

void OpPlan::drop_graph() {
  if (gexec_) cudaGraphExecDestroy(gexec_);
  gexec_ = nullptr;
  if (cap_stream_) cudaStreamDestroy(cap_stream_);
  cap_stream_ = nullptr;
}

void OpPlan::clear() {
  drop_graph();
  seq_.clear();
  gemm_.clear();
  gemm_flops_.clear();
  attn_.clear();
  gn_.clear();
  ln_.clear();
  custom_.clear();
  custom_flops_.clear();
}

void OpPlan::push_gemm(const GemmOp& g, double flops) {
  gemm_.push_back(g);
  gemm_flops_.push_back(flops >= 0.0 ? flops : 2.0 * g.p.M * static_cast<double>(g.p.N) * g.k_true);
  seq_.push_back({Kind::Gemm, static_cast<int>(gemm_.size() - 1)});
}
void OpPlan::push_attn(const AttnOp& a) {
  attn_.push_back(a);
  seq_.push_back({Kind::Attn, static_cast<int>(attn_.size() - 1)});
}
void OpPlan::push_gn(const GnOp& g) {
  gn_.push_back(g);
  seq_.push_back({Kind::Gn, static_cast<int>(gn_.size() - 1)});
}
void OpPlan::push_ln(const LnArgs& l) {
  ln_.push_back(l);
  seq_.push_back({Kind::Ln, static_cast<int>(ln_.size() - 1)});
}
void OpPlan::push_custom(std::function<int(cudaStream_t)> f, double flops) {
  custom_.push_back(std::move(f));
  custom_flops_.push_back(flops);
  seq_.push_back({Kind::Custom, static_cast<int>(custom_.size() - 1)});
}

int OpPlan::num_launches() const {
  int n = 0;
  for (const auto& o : seq_) n += o.kind == Kind::Gn ? 2 : 1;
  return n;
}

int OpPlan::launch(const Ref& o, cudaStream_t s) {
  switch (o.kind) {
    case Kind::Gemm: return gemm_launch(gemm_[o.idx], s);
    case Kind::Attn: return attn_launch(attn_[o.idx], s);
    case Kind::Gn: return gn_launch(gn_[o.idx], s);
    case Kind::Ln: {
      const LnArgs& l = ln_[o.idx];
      return layer_norm(l.x, l.g, l.b, l.out, l.rows, l.C, l.eps, s);
    }
    case Kind::Custom: return custom_[o.idx](s);
  }
  return DLM_ERR_INVALID;
}

int OpPlan::run(cudaStream_t s) {
  for (const Ref& o : seq_) {
    const int rc = launch(o, s);
    if (rc != DLM_OK) return rc;
  }
  return DLM_OK;
}

int OpPlan::replay(cudaStream_t s, bool graph) {
  if (!graph) return run(s);
  if (!gexec_) {
    if (!cap_stream_) DLM_CHECK_CUDA(cudaStreamCreateWithFlags(&cap_stream_, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    DLM_CHECK_CUDA(cudaStreamBeginCapture(cap_stream_, cudaStreamCaptureModeThreadLocal));
    const int rc = run(cap_stream_);
    cudaError_t ce = cudaStreamEndCapture(cap_stream_, &g);
    if (rc != DLM_OK) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    DLM_CHECK_CUDA(ce);
    ce = cudaGraphInstantiate(&gexec_, g, 0);
    cudaGraphDestroy(g);
    DLM_CHECK_CUDA(ce);
  }
  DLM_CHECK_CUDA(cudaGraphLaunch(gexec_, s));
  return DLM_OK;
}

int OpPlan::time(cudaStream_t s, double* ms, double* flops, int* count) {
  for (int k = 0; k < kNumClasses; ++k) {
    ms[k] = 0.0;
    flops[k] = 0.0;
    count[k] = 0;
  }
  const char* table_path = std::getenv("DLM_OP_TABLE");
  FILE* table = table_path ? std::fopen(table_path, "w") : nullptr;
  if (table) std::fprintf(table, "kind,M,N,K,bn,pair,amode,flags,us\n");
  std::vector<cudaEvent_t> ev(seq_.size() + 1, nullptr);
  int rc = DLM_OK;
  for (auto& e : ev)
    if (cudaEventCreate(&e) != cudaSuccess) rc = DLM_ERR_CUDA;
  if (rc == DLM_OK && cudaEventRecord(ev[0], s) != cudaSuccess) rc = DLM_ERR_CUDA;
  for (size_t i = 0; i < seq_.size() && rc == DLM_OK; ++i) {
    rc = launch(seq_[i], s);
    if (rc == DLM_OK && cudaEventRecord(ev[i + 1], s) != cudaSuccess) rc = DLM_ERR_CUDA;
  }
  if (rc == DLM_OK && cudaStreamSynchronize(s) != cudaSuccess) rc = DLM_ERR_CUDA;
  for (size_t i = 0; i < seq_.size() && rc == DLM_OK; ++i) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
    const Ref& o = seq_[i];
    int k = 4;
    double f = 0.0;
    if (o.kind == Kind::Gemm) {
      k = 0;
      f = gemm_flops_[o.idx];
    } else if (o.kind == Kind::Attn) {
      k = 1;
      const AttnParams& p = attn_[o.idx].p;
      f = 4.0 * p.B * p.H * static_cast<double>(p.Sq) * p.Sk * 64;
    } else if (o.kind == Kind::Gn) {
      k = 2;
    } else if (o.kind == Kind::Ln) {
      k = 3;
    } else {
      f = custom_flops_[o.idx];
    }
    ms[k] += t;
    flops[k] += f;
    count[k] += o.kind == Kind::Gn ? 2 : 1;
    if (table) {
      // one line per launch: class, shape, tile choice, epilogue flags, microseconds
      if (o.kind == Kind::Gemm) {
        const GemmOp& g = gemm_[o.idx];
        std::fprintf(table, "gemm,%d,%d,%lld,%d,%d,%d,0x%x,%.2f\n", g.p.M, g.p.N, g.k_true, g.bn,
                     g.pair ? 1 : 0, g.p.amode, g.p.flags, 1000.0 * t);
      } else if (o.kind == Kind::Attn) {
        const AttnParams& a = attn_[o.idx].p;
        std::fprintf(table, "attn,%d,%d,%d,%d,0,0,0,%.2f\n", a.B * a.H, a.Sq, a.Sk, 64, 1000.0 * t);
      } else {
        std::fprintf(table, "%s,0,0,0,0,0,0,0,%.2f\n",
                     o.kind == Kind::Gn ? "groupnorm" : o.kind == Kind::Ln ? "layernorm" : "other",
                     1000.0 * t);
      }
    }
  }
  if (table) std::fclose(table);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

}  // namespace dlm
