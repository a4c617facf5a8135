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
  attn_wide_.clear();
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
void OpPlan::push_attn_wide(const AttnWideOp& a) {
  attn_wide_.push_back(a);
  seq_.push_back({Kind::AttnWide, static_cast<int>(attn_wide_.size() - 1)});
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
    case Kind::AttnWide: return attn_wide_launch(attn_wide_[o.idx], s);
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

int OpPlan::op_class(const Ref& o, double* f) const {
  switch (o.kind) {
    case Kind::Gemm: *f = gemm_flops_[o.idx]; return 0;
    case Kind::Attn: {
      const AttnParams& p = attn_[o.idx].p;
      *f = 4.0 * p.B * p.H * static_cast<double>(p.Sq) * p.Sk * 64;
      return 1;
    }
    case Kind::AttnWide: {
      const AttnWideParams& p = attn_wide_[o.idx].p;
      *f = 4.0 * p.B * p.H * static_cast<double>(p.Sq) * p.Sk * p.Dh;
      return 1;
    }
    case Kind::Gn: *f = 0.0; return 2;
    case Kind::Ln: *f = 0.0; return 3;
    case Kind::Custom: *f = custom_flops_[o.idx]; return 4;
  }
  *f = 0.0;
  return 4;
}

// One line per launch of an eager step with an event between launches (DLM_OP_TABLE): class,
// shape, tile choice, epilogue flags, microseconds.  Diagnostic only: the events between
// launches stretch every launch by a few microseconds.
int OpPlan::write_table(cudaStream_t s, const char* path) {
  FILE* table = std::fopen(path, "w");
  if (!table) return DLM_OK;
  std::fprintf(table, "kind,M,N,K,bn,pair,amode,flags,us\n");
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
    if (o.kind == Kind::Gemm) {
      const GemmOp& g = gemm_[o.idx];
      std::fprintf(table, "gemm,%d,%d,%lld,%d,%d,%d,0x%x,%.2f\n", g.p.M, g.p.N, g.k_true, g.bn,
                   g.pair ? 1 : 0, g.p.amode, g.p.flags, 1000.0 * t);
    } else if (o.kind == Kind::Attn) {
      const AttnParams& a = attn_[o.idx].p;
      std::fprintf(table, "attn,%d,%d,%d,%d,0,0,0,%.2f\n", a.B * a.H, a.Sq, a.Sk, 64, 1000.0 * t);
    } else if (o.kind == Kind::AttnWide) {
      const AttnWideParams& a = attn_wide_[o.idx].p;
      std::fprintf(table, "attn,%d,%d,%d,%d,0,0,0,%.2f\n", a.B * a.H, a.Sq, a.Sk, a.Dh, 1000.0 * t);
    } else {
      std::fprintf(table, "%s,0,0,0,0,0,0,0,%.2f\n",
                   o.kind == Kind::Gn ? "groupnorm" : o.kind == Kind::Ln ? "layernorm" : "other",
                   1000.0 * t);
    }
  }
  std::fclose(table);
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  return rc;
}

// Per class: the class's launches alone (in step order) captured as one CUDA graph and replayed
// kReps times between two events, so a class's time has the same launch overheads and overlap
// between consecutive kernels as inside the step graph, and the classes' times add up to about
// the step's.  Inputs of a class's kernels are whatever the previous step left in the arena
// (finite values); every counter / flag the kernels use is left at zero by each launch.
int OpPlan::time(cudaStream_t s, double* ms, double* flops, int* count) {
  constexpr int kReps = 5;
  std::vector<int> cls(seq_.size());
  for (int k = 0; k < kNumClasses; ++k) {
    ms[k] = 0.0;
    flops[k] = 0.0;
    count[k] = 0;
  }
  for (size_t i = 0; i < seq_.size(); ++i) {
    double f = 0.0;
    cls[i] = op_class(seq_[i], &f);
    flops[cls[i]] += f;
    count[cls[i]] += seq_[i].kind == Kind::Gn ? 2 : 1;
  }
  if (const char* table_path = std::getenv("DLM_OP_TABLE")) {
    const int rc = write_table(s, table_path);
    if (rc != DLM_OK) return rc;
  }
  if (!cap_stream_) DLM_CHECK_CUDA(cudaStreamCreateWithFlags(&cap_stream_, cudaStreamNonBlocking));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  DLM_CHECK_CUDA(cudaEventCreate(&e0));
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return DLM_ERR_CUDA;
  }
  int rc = DLM_OK;
  for (int k = 0; k < kNumClasses && rc == DLM_OK; ++k) {
    if (count[k] == 0) continue;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    if (cudaStreamBeginCapture(cap_stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      rc = DLM_ERR_CUDA;
      break;
    }
    for (size_t i = 0; i < seq_.size() && rc == DLM_OK; ++i)
      if (cls[i] == k) rc = launch(seq_[i], cap_stream_);
    const cudaError_t ce = cudaStreamEndCapture(cap_stream_, &g);
    if (rc == DLM_OK && ce != cudaSuccess) rc = DLM_ERR_CUDA;
    if (rc == DLM_OK && cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) rc = DLM_ERR_CUDA;
    if (g) cudaGraphDestroy(g);
    if (rc == DLM_OK && cudaGraphLaunch(ge, s) != cudaSuccess) rc = DLM_ERR_CUDA;  // warm-up
    if (rc == DLM_OK && cudaEventRecord(e0, s) != cudaSuccess) rc = DLM_ERR_CUDA;
    for (int r = 0; r < kReps && rc == DLM_OK; ++r)
      if (cudaGraphLaunch(ge, s) != cudaSuccess) rc = DLM_ERR_CUDA;
    if (rc == DLM_OK && cudaEventRecord(e1, s) != cudaSuccess) rc = DLM_ERR_CUDA;
    if (rc == DLM_OK && cudaEventSynchronize(e1) != cudaSuccess) rc = DLM_ERR_CUDA;
    float t = 0.0f;
    if (rc == DLM_OK && cudaEventElapsedTime(&t, e0, e1) != cudaSuccess) rc = DLM_ERR_CUDA;
    ms[k] = static_cast<double>(t) / kReps;
    if (ge) cudaGraphExecDestroy(ge);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return rc;
}

}  // namespace dlm
