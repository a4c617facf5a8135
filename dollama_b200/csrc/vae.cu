// SDXL AutoencoderKL decoder on the B200 kernels (host orchestration, C++).
//
// Replaces the reference's VAE decoder (src/kernels/vae_decode.cu: launch_vae_decode_impl :699,
// resnet_block :621, resnet_block_f32 :575, attn_block :660) and its weight handle
// (vae_weights_create :894, launch_vae_decode(handle, ...) vae_decode.cuh:73-75), behind dlm_vae_*
// in the C ABI.
//
// Design (B200-first, not a translation):
//   * activations are NHWC end to end; every conv is the implicit-GEMM tcgen05 kernel with the
//     bias, the identity residual and the 1x1 conv_shortcut (extra K segment) fused, so a
//     ResnetBlock is GN -> conv1 -> GN -> conv2 (4 launches of which 2 GroupNorm pairs);
//   * the numerics follow the reference's split: fp16 activations up to up_blocks[1], fp32
//     activations ("carries") from up_blocks[2] on, because those residual blocks leave the fp16
//     range (vae_decode.cu:9-20).  The fp32 carries never enter a GEMM as fp32: GroupNorm reads
//     them in fp32 and writes its normalised fp16 output, the GEMM epilogue adds the fp32 residual
//     and stores fp32, and where a raw carry is a GEMM operand (the up_blocks[2] upsampler input,
//     up_blocks[3].resnets.0's conv_shortcut input) it is converted to fp16 divided by 64 and the
//     64 is restored exactly (a power of two) in the epilogue's alpha or in the packed shortcut
//     weights.  fp16 operands carry the same 10-bit mantissa as the reference's default TF32
//     GEMMs, with fp32 accumulation;
//   * the mid-block attention (one head, Dh = 512, S = h*w tokens) is one wide-head flash
//     attention launch over the batch (attention_wide.cu): fp32 online softmax, unnormalised fp16
//     P, the row-sum division on the fp32 accumulator, no S x S scores in memory;
//   * the whole decode is planned once per latent shape over one static arena and replays as one
//     CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "gemm.h"
#include "norm.h"
#include "ops.h"
#include "vae.h"

namespace dlm {

namespace {

constexpr int kLatC = 4;
constexpr int kLatPad = 64;   // latent channels padded to one 64-channel K block
constexpr int kTop = 512;     // channels of the mid block and up_blocks[0..1]
constexpr int kUpC[4] = {512, 512, 256, 128};
constexpr int kOutPad = 32;   // conv_out's 3 output channels padded to one 32-column chunk
constexpr float kEps = 1e-6f;
constexpr float kCarryScale = 64.0f;

// w[r * ld + c] *= s for r < rows, c < cols (power-of-two scale: exact for normal fp16 values)
__global__ void scale_block_kernel(__half* w, int rows, int cols, int ld, float s) {
  const size_t total = static_cast<size_t>(rows) * cols;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / cols, c = i % cols;
    __half* p = w + r * ld + c;
    *p = __float2half_rn(__half2float(*p) * s);
  }
}

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto d : s) n *= d;
  return n;
}

std::string up_resnet(int u, int r) {
  return "decoder.up_blocks." + std::to_string(u) + ".resnets." + std::to_string(r) + ".";
}
std::string up_sampler(int u) {
  return "decoder.up_blocks." + std::to_string(u) + ".upsamplers.0.conv";
}

}  // namespace

// Weight names and shapes of the diffusers AutoencoderKL state dict the reference loads
// (decoder.* and post_quant_conv.*; 140 tensors).
std::vector<VaeWeightSpec> vae_weight_specs() {
  std::vector<VaeWeightSpec> S;
  auto cv = [&](const std::string& n, int o, int i, int k = 3) {
    S.push_back({n + ".weight", {o, i, k, k}});
    S.push_back({n + ".bias", {o}});
  };
  auto nrm = [&](const std::string& n, int c) {
    S.push_back({n + ".weight", {c}});
    S.push_back({n + ".bias", {c}});
  };
  auto res = [&](const std::string& p, int cin, int cout) {
    nrm(p + "norm1", cin);
    cv(p + "conv1", cout, cin);
    nrm(p + "norm2", cout);
    cv(p + "conv2", cout, cout);
    if (cin != cout) cv(p + "conv_shortcut", cout, cin, 1);
  };
  cv("post_quant_conv", kLatC, kLatC, 1);
  cv("decoder.conv_in", kTop, kLatC);
  res("decoder.mid_block.resnets.0.", kTop, kTop);
  const std::string a = "decoder.mid_block.attentions.0.";
  nrm(a + "group_norm", kTop);
  for (const char* n : {"to_q", "to_k", "to_v", "to_out.0"}) {
    S.push_back({a + n + ".weight", {kTop, kTop}});
    S.push_back({a + n + ".bias", {kTop}});
  }
  res("decoder.mid_block.resnets.1.", kTop, kTop);
  int cin = kTop;
  for (int u = 0; u < 4; ++u) {
    for (int r = 0; r < 3; ++r) res(up_resnet(u, r), r == 0 ? cin : kUpC[u], kUpC[u]);
    cin = kUpC[u];
    if (u < 3) cv(up_sampler(u), kUpC[u], kUpC[u]);
  }
  nrm("decoder.conv_norm_out", kUpC[3]);
  cv("decoder.conv_out", 3, kUpC[3]);
  return S;
}

VAEModel::~VAEModel() {
  release_plan();
  if (wbuf_) cudaFree(wbuf_);
}

void VAEModel::release_plan() {
  ops_.clear();
  if (abuf_) cudaFree(abuf_);
  abuf_ = nullptr;
  B_ = h_ = w_lat_ = 0;
  stages_.clear();
}

__half* VAEModel::wtake(size_t elems) {
  const size_t bytes = ((elems * 2 + 255) / 256) * 256;
  if (woff_ + bytes > wcap_) return nullptr;
  __half* p = reinterpret_cast<__half*>(static_cast<char*>(wbuf_) + woff_);
  woff_ += bytes;
  return p;
}

const __half* VAEModel::src(const std::string& n) const {
  auto it = src_.find(n);
  return it == src_.end() ? nullptr : it->second;
}

const __half* VAEModel::W(const std::string& n) const {
  auto it = w_.find(n);
  return it == w_.end() ? nullptr : it->second;
}

int VAEModel::create(int n, const char* const* names, const void* const* ptrs,
                     const int64_t* numels, cudaStream_t s) {
  const auto specs = vae_weight_specs();
  std::unordered_map<std::string, std::pair<const __half*, int64_t>> given;
  for (int i = 0; i < n; ++i) {
    DLM_REQUIRE(names[i] != nullptr && ptrs[i] != nullptr, DLM_ERR_INVALID,
                "vae_create: null name or pointer at %d", i);
    given[names[i]] = {static_cast<const __half*>(ptrs[i]), numels ? numels[i] : -1};
  }
  size_t total = 0;
  for (const auto& sp : specs) {
    auto it = given.find(sp.name);
    DLM_REQUIRE(it != given.end(), DLM_ERR_NOT_FOUND, "vae_create: missing weight %s",
                sp.name.c_str());
    DLM_REQUIRE(it->second.second < 0 || it->second.second == numel(sp.shape), DLM_ERR_INVALID,
                "vae_create: %s has %lld elements, expected %lld", sp.name.c_str(),
                static_cast<long long>(it->second.second), static_cast<long long>(numel(sp.shape)));
    src_[sp.name] = it->second.first;
    total += static_cast<size_t>(numel(sp.shape)) * 2 + 512;
  }
  // padded post_quant_conv / conv_in / conv_out layouts
  total += (static_cast<size_t>(kLatPad) * kLatPad + static_cast<size_t>(kTop) * 9 * kLatPad +
            static_cast<size_t>(kOutPad) * 9 * kUpC[3] + 4096) * 2;
  wcap_ = total;
  DLM_CHECK_CUDA(cudaMalloc(&wbuf_, wcap_));
  woff_ = 0;
  int rc = prepare_weights(s);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  src_.clear();  // the caller's buffers are no longer referenced
  return DLM_OK;
}

// Copies / repacks every weight into the layouts the kernels read: convs as [Cout, tap, Cin]
// (conv2 and its 1x1 conv_shortcut side by side in one K range, biases summed), q/k/v concatenated.
int VAEModel::prepare_weights(cudaStream_t s) {
  auto fail = [&](const char* what) {
    set_error("vae prepare: %s", what);
    return DLM_ERR_NOMEM;
  };
  auto copy = [&](const std::string& name, size_t elems) -> __half* {
    __half* d = wtake(elems);
    if (!d) return nullptr;
    if (cudaMemcpyAsync(d, src(name), elems * 2, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return nullptr;
    w_[name] = d;
    return d;
  };
  // packed conv weight (+ bias, optionally zero-padded rows)
  auto conv = [&](const std::string& p, int cout, int cout_pad, int cin, int cin_pad, int kk) -> int {
    __half* d = wtake(static_cast<size_t>(cout_pad) * kk * cin_pad);
    __half* b = wtake(cout_pad);
    if (!d || !b) return fail(p.c_str());
    int rc = pack_conv_pad(src(p + ".weight"), d, cout, cout_pad, cin, cin_pad, kk, kk * cin_pad, s);
    if (rc != DLM_OK) return rc;
    if (cout_pad != cout) DLM_CHECK_CUDA(cudaMemsetAsync(b, 0, cout_pad * 2, s));
    DLM_CHECK_CUDA(cudaMemcpyAsync(b, src(p + ".bias"), cout * 2, cudaMemcpyDeviceToDevice, s));
    w_[p + ".packed"] = d;
    w_[p + ".bias"] = b;
    return DLM_OK;
  };
  // shortcut_scale: the conv_shortcut input arrives divided by it (an fp32 carry as fp16 / 64)
  auto resnet = [&](const std::string& p, int ci, int co, float shortcut_scale) -> int {
    for (const char* nn : {"norm1.weight", "norm1.bias"})
      if (!copy(p + nn, ci)) return fail("resnet norm1");
    for (const char* nn : {"norm2.weight", "norm2.bias"})
      if (!copy(p + nn, co)) return fail("resnet norm2");
    int rc = conv(p + "conv1", co, co, ci, ci, 9);
    if (rc != DLM_OK) return rc;
    const bool sc = ci != co;
    const int k2 = 9 * co + (sc ? ci : 0);
    __half* w2 = wtake(static_cast<size_t>(co) * k2);
    __half* b2 = wtake(co);
    if (!w2 || !b2) return fail("conv2");
    rc = pack_conv_pad(src(p + "conv2.weight"), w2, co, co, co, co, 9, k2, s);
    if (rc != DLM_OK) return rc;
    if (sc) {
      DLM_CHECK_CUDA(cudaMemcpy2DAsync(w2 + 9 * co, static_cast<size_t>(k2) * 2,
                                       src(p + "conv_shortcut.weight"), static_cast<size_t>(ci) * 2,
                                       static_cast<size_t>(ci) * 2, co, cudaMemcpyDeviceToDevice, s));
      if (shortcut_scale != 1.0f) {
        scale_block_kernel<<<256, 256, 0, s>>>(w2 + 9 * co, co, ci, k2, shortcut_scale);
        DLM_CHECK_CUDA(cudaGetLastError());
      }
      rc = add_f16(src(p + "conv2.bias"), src(p + "conv_shortcut.bias"), b2, co, s);
      if (rc != DLM_OK) return rc;
    } else {
      DLM_CHECK_CUDA(cudaMemcpyAsync(b2, src(p + "conv2.bias"), co * 2, cudaMemcpyDeviceToDevice, s));
    }
    w_[p + "conv2.packed"] = w2;
    w_[p + "conv2.bias_f"] = b2;
    return DLM_OK;
  };

  int rc = conv("post_quant_conv", kLatC, kLatPad, kLatC, kLatPad, 1);
  if (rc == DLM_OK) rc = conv("decoder.conv_in", kTop, kTop, kLatC, kLatPad, 9);
  if (rc == DLM_OK) rc = resnet("decoder.mid_block.resnets.0.", kTop, kTop, 1.0f);
  if (rc == DLM_OK) rc = resnet("decoder.mid_block.resnets.1.", kTop, kTop, 1.0f);
  if (rc != DLM_OK) return rc;
  {
    const std::string a = "decoder.mid_block.attentions.0.";
    for (const char* nn : {"group_norm.weight", "group_norm.bias"})
      if (!copy(a + nn, kTop)) return fail("attention group_norm");
    const size_t mat = static_cast<size_t>(kTop) * kTop;
    __half* qkv = wtake(3 * mat);
    __half* qkvb = wtake(3 * kTop);
    if (!qkv || !qkvb) return fail("attention qkv");
    const char* parts[3] = {"to_q", "to_k", "to_v"};
    for (int i = 0; i < 3; ++i) {
      DLM_CHECK_CUDA(cudaMemcpyAsync(qkv + i * mat, src(a + parts[i] + ".weight"), mat * 2,
                                     cudaMemcpyDeviceToDevice, s));
      DLM_CHECK_CUDA(cudaMemcpyAsync(qkvb + i * kTop, src(a + parts[i] + ".bias"), kTop * 2,
                                     cudaMemcpyDeviceToDevice, s));
    }
    w_[a + "qkv.weight"] = qkv;
    w_[a + "qkv.bias"] = qkvb;
    if (!copy(a + "to_out.0.weight", mat) || !copy(a + "to_out.0.bias", kTop))
      return fail("attention to_out");
  }
  int cin = kTop;
  for (int u = 0; u < 4 && rc == DLM_OK; ++u) {
    for (int r = 0; r < 3 && rc == DLM_OK; ++r) {
      const int ci = r == 0 ? cin : kUpC[u];
      // up_blocks[3].resnets[0] is the only block whose conv_shortcut reads an fp32 carry
      rc = resnet(up_resnet(u, r), ci, kUpC[u], (u == 3 && r == 0) ? kCarryScale : 1.0f);
    }
    cin = kUpC[u];
    if (u < 3 && rc == DLM_OK) rc = conv(up_sampler(u), kUpC[u], kUpC[u], kUpC[u], kUpC[u], 9);
  }
  if (rc != DLM_OK) return rc;
  for (const char* nn : {"decoder.conv_norm_out.weight", "decoder.conv_norm_out.bias"})
    if (!copy(nn, kUpC[3])) return fail("conv_norm_out");
  rc = conv("decoder.conv_out", 3, kOutPad, kUpC[3], kUpC[3], 9);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaGetLastError());
  return DLM_OK;
}

// ================================================================== plan

#define PLAN_CHECK(expr)             \
  do {                               \
    if (!dry_) {                     \
      int _rc = (expr);              \
      if (_rc != DLM_OK) return _rc; \
    }                                \
  } while (0)

int VAEModel::plan_gn(const Act& x, int HW, const std::string& wprefix, bool silu, __half* out) {
  if (dry_) return DLM_OK;
  GnOp g;
  int rc = x.f32 ? gn_plan_f32(&g, static_cast<const float*>(x.p), x.C, B_, HW, W(wprefix + ".weight"),
                               W(wprefix + ".bias"), kEps, silu, out, gn_partials_, gn_partial_cap_)
                 : gn_plan(&g, static_cast<const __half*>(x.p), x.C, nullptr, 0, B_, HW,
                           W(wprefix + ".weight"), W(wprefix + ".bias"), kEps, silu, out,
                           gn_partials_, gn_partial_cap_);
  if (rc != DLM_OK) return rc;
  ops_.push_gn(g);
  return DLM_OK;
}

// ResnetBlock2D (vae_decode.cu:621-658, fp32 form :575-619):
//   out = conv2(silu(GN(conv1(silu(GN(x)))))) + (x | conv_shortcut(x))
// conv1 stores fp32 when the block's output is an fp32 carry; conv2, the shortcut K segment, the
// summed biases and the identity residual are one GEMM.
int VAEModel::plan_resnet(const std::string& p, const Act& x, int cout, int H, int Wd, const Act& out) {
  const int HW = H * Wd;
  const size_t P = static_cast<size_t>(B_) * HW;
  int rc = plan_gn(x, HW, p + "norm1", true, s_gn1_);
  if (rc != DLM_OK) return rc;
  const Act c1{s_c1_, out.f32, cout};
  if (!dry_) {
    GemmOp g;
    ConvSource s0{0, s_gn1_, x.C};
    GemmEpilogue e;
    e.flags = DLM_EPI_BIAS | (out.f32 ? kEpiOutF32 : 0u);
    e.bias = W(p + "conv1.bias");
    rc = gemm_plan_conv(&g, B_, H, Wd, &s0, 1, W(p + "conv1.packed"), cout,
                        static_cast<__half*>(c1.p), cout, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g);
  }
  rc = plan_gn(c1, HW, p + "norm2", true, s_gn2_);
  if (rc != DLM_OK) return rc;
  if (x.C != cout && x.f32 && !dry_) {
    // the shortcut operand: the fp32 carry as fp16 / 64 (the packed shortcut weights carry the 64)
    const float* xf = static_cast<const float*>(x.p);
    __half* xs = upbuf_;
    const size_t n = P * x.C;
    ops_.push_custom([=](cudaStream_t s) { return f32_to_f16_scaled(xf, xs, n, 1.0f / kCarryScale, s); });
  }
  if (!dry_) {
    GemmOp g;
    ConvSource srcs[2];
    int ns = 0;
    srcs[ns++] = ConvSource{0, s_gn2_, cout};
    GemmEpilogue e;
    e.flags = DLM_EPI_BIAS | (out.f32 ? kEpiOutF32 : 0u);
    e.bias = W(p + "conv2.bias_f");
    if (x.C != cout) {
      srcs[ns++] = ConvSource{1, x.f32 ? upbuf_ : static_cast<const __half*>(x.p), x.C};
    } else {
      e.flags |= DLM_EPI_RESID | (x.f32 ? kEpiResidF32 : 0u);
      e.resid = static_cast<const __half*>(x.p);
      e.ldr = cout;
    }
    rc = gemm_plan_conv(&g, B_, H, Wd, srcs, ns, W(p + "conv2.packed"), cout,
                        static_cast<__half*>(out.p), cout, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g);
  }
  return DLM_OK;
}

// Mid-block AttnBlock (vae_decode.cu:660-691), in place on x [B*S, 512] fp16:
//   x += to_out(softmax(q k^T / sqrt(512)) v),  q|k|v = GN(x) Wqkv^T + b  (one GEMM)
int VAEModel::plan_attn(const std::string& p, const Act& x, int H, int Wd) {
  const int S = H * Wd, M = B_ * S, C = kTop;
  int rc = plan_gn(x, S, p + "group_norm", false, s_gn1_);
  if (rc != DLM_OK) return rc;
  if (dry_) return DLM_OK;
  __half* xh = static_cast<__half*>(x.p);
  {
    GemmOp g;
    GemmEpilogue e;
    e.flags = DLM_EPI_BIAS;
    e.bias = W(p + "qkv.bias");
    rc = gemm_plan_dense(&g, s_gn1_, C, W(p + "qkv.weight"), M, 3 * C, C, qkv_, 3 * C, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g);
  }
  {
    // one wide-head flash attention over the B images: q | k | v token-major [B*S, 3C] (one
    // head of C = 512 columns), out [B*S, C]
    auto tok = [&](const __half* ptr, long long ld) {
      AttnTensor t;
      t.ptr = ptr;
      t.ss = ld;
      t.sh = C;
      t.sb = static_cast<long long>(S) * ld;
      return t;
    };
    AttnWideOp a;
    rc = attn_wide_plan(&a, B_, 1, S, S, C, 1.0f / std::sqrt(static_cast<float>(C)),
                        tok(qkv_, 3 * C), tok(qkv_ + C, 3 * C), tok(qkv_ + 2 * C, 3 * C),
                        tok(attn_o_, C));
    if (rc != DLM_OK) return rc;
    ops_.push_attn_wide(a);
  }
  GemmOp g;
  GemmEpilogue e;
  e.flags = DLM_EPI_BIAS | DLM_EPI_RESID;
  e.bias = W(p + "to_out.0.bias");
  e.resid = xh;
  e.ldr = C;
  rc = gemm_plan_dense(&g, attn_o_, C, W(p + "to_out.0.weight"), M, C, C, xh, C, e);
  if (rc != DLM_OK) return rc;
  ops_.push_gemm(g);
  return DLM_OK;
}

// nearest 2x upsample + 3x3 conv (vae_decode.cu:777-787); an fp32 input is converted to fp16 / 64
// on the way and the conv's epilogue multiplies the 64 back.
int VAEModel::plan_upsample(const std::string& p, const Act& x, int H, int Wd, const Act& out) {
  if (dry_) return DLM_OK;
  const int C = x.C;
  const int B = B_;
  __half* up = upbuf_;
  float alpha = 1.0f;
  if (x.f32) {
    const float* xf = static_cast<const float*>(x.p);
    ops_.push_custom([=](cudaStream_t s) {
      return upsample2x_f32_to_f16(xf, up, B, H, Wd, C, 1.0f / kCarryScale, s);
    });
    alpha = kCarryScale;
  } else {
    const __half* xh = static_cast<const __half*>(x.p);
    ops_.push_custom([=](cudaStream_t s) { return upsample2x_nhwc(xh, up, B, H, Wd, C, s); });
  }
  GemmOp g;
  ConvSource s0{0, upbuf_, C};
  GemmEpilogue e;
  e.flags = DLM_EPI_BIAS | (out.f32 ? kEpiOutF32 : 0u);
  e.alpha = alpha;
  e.bias = W(p + ".bias");
  int rc = gemm_plan_conv(&g, B, 2 * H, 2 * Wd, &s0, 1, W(p + ".packed"), C,
                          static_cast<__half*>(out.p), C, e);
  if (rc != DLM_OK) return rc;
  ops_.push_gemm(g);
  return DLM_OK;
}

int VAEModel::build(bool dry) {
  dry_ = dry;
  arena_.begin(dry, abuf_);
  ops_.clear();
  stages_.clear();
  const int B = B_;
  int Hs[4], Ws[4];
  size_t P[4];
  for (int l = 0; l < 4; ++l) {
    Hs[l] = h_ << l;
    Ws[l] = w_lat_ << l;
    P[l] = static_cast<size_t>(B) * Hs[l] * Ws[l];
  }
  const int S = h_ * w_lat_;
  auto f16 = [&](size_t px, int c) { return Act{arena_.take<__half>(px * c), false, c}; };
  auto f32 = [&](size_t px, int c) { return Act{arena_.take<float>(px * c), true, c}; };

  lat_in_ = arena_.take<__half>(static_cast<size_t>(B) * kLatC * S);
  image_ = arena_.take<__half>(P[3] * 3);
  lat64_ = arena_.take<__half>(P[0] * kLatPad);
  pqc_ = arena_.take<__half>(P[0] * kLatPad);
  const Act x0 = f16(P[0], kTop), m0 = f16(P[0], kTop), mid_out = f16(P[0], kTop);
  const Act l0a = f16(P[0], kTop), l0b = f16(P[0], kTop), up0_out = f16(P[1], kTop);
  const Act l1a = f16(P[1], kTop), l1b = f16(P[1], kTop), up1_out = f16(P[2], kTop);
  const Act l2a = f32(P[2], kUpC[2]), l2b = f32(P[2], kUpC[2]), up2_out = f32(P[3], kUpC[2]);
  const Act l3a = f32(P[3], kUpC[3]), l3b = f32(P[3], kUpC[3]), up3_out = f32(P[3], kUpC[3]);
  s_gn1_ = arena_.take<__half>(std::max({P[1] * kTop, P[2] * kTop, P[3] * kUpC[2]}));
  s_c1_ = arena_.take<char>(std::max({P[1] * kTop * 2, P[2] * kUpC[2] * 4, P[3] * kUpC[3] * 4}));
  s_gn2_ = arena_.take<__half>(std::max({P[1] * kTop, P[2] * kUpC[2], P[3] * kUpC[3]}));
  upbuf_ = arena_.take<__half>(std::max({P[1] * kTop, P[2] * kTop, P[3] * kUpC[2]}));
  out32_ = arena_.take<__half>(P[3] * kOutPad);
  qkv_ = arena_.take<__half>(P[0] * 3 * kTop);
  attn_o_ = arena_.take<__half>(P[0] * kTop);
  gn_partial_cap_ = gn_partial_elems(B, Hs[3] * Ws[3]);
  gn_partials_ = arena_.take<float2>(gn_partial_cap_);

  // post_quant_conv (1x1) and conv_in (3x3) on the latent padded to 64 channels
  if (!dry_) {
    const __half* li = lat_in_;
    __half* l64 = lat64_;
    ops_.push_custom([=](cudaStream_t s) { return nchw_to_nhwc_pad(li, l64, B, kLatC, S, kLatPad, s); });
    GemmOp g;
    ConvSource s0{1, lat64_, kLatPad};
    GemmEpilogue e;
    e.flags = DLM_EPI_BIAS;
    e.bias = W("post_quant_conv.bias");
    int rc = gemm_plan_conv(&g, B, h_, w_lat_, &s0, 1, W("post_quant_conv.packed"), kLatPad, pqc_,
                            kLatPad, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g, 2.0 * P[0] * kLatC * kLatC);
    ConvSource s1{0, pqc_, kLatPad};
    e.bias = W("decoder.conv_in.bias");
    rc = gemm_plan_conv(&g, B, h_, w_lat_, &s1, 1, W("decoder.conv_in.packed"), kTop,
                        static_cast<__half*>(x0.p), kTop, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g, 2.0 * P[0] * kLatC * 9 * kTop);
  }
  auto stage = [&](const char* name, const Act& a, int l) {
    stages_[name] = StageInfo{a.p, a.f32 ? 1 : 0, a.C, Hs[l], Ws[l]};
  };
  int rc = plan_resnet("decoder.mid_block.resnets.0.", x0, kTop, h_, w_lat_, m0);
  if (rc == DLM_OK) rc = plan_attn("decoder.mid_block.attentions.0.", m0, h_, w_lat_);
  if (rc == DLM_OK) rc = plan_resnet("decoder.mid_block.resnets.1.", m0, kTop, h_, w_lat_, mid_out);
  if (rc != DLM_OK) return rc;
  stage("mid_block_out", mid_out, 0);
  // up_blocks: three resnets ping-ponging between two level buffers, then the upsampler into the
  // next level's input (up_blocks[3] has none: its last resnet writes the stage buffer)
  const Act ins[4] = {mid_out, up0_out, up1_out, up2_out};
  const Act pa[4] = {l0a, l1a, l2a, l3a}, pb[4] = {l0b, l1b, l2b, l3b};
  const Act outs[4] = {up0_out, up1_out, up2_out, up3_out};
  for (int u = 0; u < 4 && rc == DLM_OK; ++u) {
    const int H = Hs[u], Wd = Ws[u];  // up_blocks[u] runs at 2^u times the latent resolution
    const Act r0 = pa[u], r1 = pb[u], r2 = u == 3 ? outs[u] : pa[u];
    rc = plan_resnet(up_resnet(u, 0), ins[u], kUpC[u], H, Wd, r0);
    if (rc == DLM_OK) rc = plan_resnet(up_resnet(u, 1), r0, kUpC[u], H, Wd, r1);
    if (rc == DLM_OK) rc = plan_resnet(up_resnet(u, 2), r1, kUpC[u], H, Wd, r2);
    if (rc == DLM_OK && u < 3) rc = plan_upsample(up_sampler(u), r2, H, Wd, outs[u]);
    const char* names[4] = {"up_block_0_out", "up_block_1_out", "up_block_2_out", "up_block_3_out"};
    stage(names[u], outs[u], u < 3 ? u + 1 : 3);
  }
  if (rc != DLM_OK) return rc;
  // conv_norm_out + SiLU (fp32 in, fp16 out) -> conv_out (128 -> 3, padded to 32) -> NCHW image
  rc = plan_gn(up3_out, Hs[3] * Ws[3], "decoder.conv_norm_out", true, s_gn1_);
  if (rc != DLM_OK) return rc;
  if (!dry_) {
    GemmOp g;
    ConvSource s0{0, s_gn1_, kUpC[3]};
    GemmEpilogue e;
    e.flags = DLM_EPI_BIAS;
    e.bias = W("decoder.conv_out.bias");
    rc = gemm_plan_conv(&g, B, Hs[3], Ws[3], &s0, 1, W("decoder.conv_out.packed"), kOutPad, out32_,
                        kOutPad, e);
    if (rc != DLM_OK) return rc;
    ops_.push_gemm(g, 2.0 * P[3] * kUpC[3] * 9 * 3);
    const __half* o32 = out32_;
    __half* img = image_;
    const int HW3 = Hs[3] * Ws[3];
    ops_.push_custom([=](cudaStream_t s) { return nhwc_to_nchw_narrow(o32, kOutPad, img, B, 3, HW3, s); });
  }
  return DLM_OK;
}

int VAEModel::plan(int B, int h, int w) {
  if (B == B_ && h == h_ && w == w_lat_ && abuf_ != nullptr) return DLM_OK;
  release_plan();
  DLM_REQUIRE(B > 0 && h > 0 && w > 0, DLM_ERR_INVALID, "vae: empty shape");
  // every conv tiles 128 output pixels as whole rows (or a multiple of rows) of one image
  const bool tiles = (w >= 128) ? (w % 128 == 0) : (128 % w == 0 && h % (128 / w) == 0);
  DLM_REQUIRE(tiles, DLM_ERR_INVALID,
              "vae: latent %dx%d: 128-pixel conv tiles need w %% 128 == 0, or w | 128 and (128 / w) | h",
              h, w);
  B_ = B;
  h_ = h;
  w_lat_ = w;
  int rc = gemm_prepare_kernels();
  if (rc != DLM_OK) return rc;
  rc = build(true);
  if (rc != DLM_OK) {
    release_plan();
    return rc;
  }
  const size_t bytes = arena_.used() + 4096;
  if (cudaMalloc(&abuf_, bytes) != cudaSuccess) {
    cudaGetLastError();
    release_plan();
    set_error("vae: cannot allocate %zu bytes of activations", bytes);
    return DLM_ERR_NOMEM;
  }
  arena_bytes_ = bytes;
  B_ = B;
  h_ = h;
  w_lat_ = w;
  rc = build(false);
  if (rc != DLM_OK) {
    release_plan();
    return rc;
  }
  // GroupNorm's arrival counters start at zero (each launch leaves them at zero)
  DLM_CHECK_CUDA(cudaMemset(gn_partials_, 0, gn_partial_cap_ * sizeof(float2)));
  DLM_CHECK_CUDA(cudaDeviceSynchronize());
  return DLM_OK;
}

int VAEModel::decode(int B, int h, int w, const __half* latent, __half* image, cudaStream_t s) {
  DLM_REQUIRE(latent && image, DLM_ERR_INVALID, "vae_decode: null input");
  int rc = plan(B, h, w);
  if (rc != DLM_OK) return rc;
  const size_t lat = static_cast<size_t>(B) * kLatC * h * w;
  const size_t img = static_cast<size_t>(B) * 3 * 64 * h * w;
  DLM_CHECK_CUDA(cudaMemcpyAsync(lat_in_, latent, lat * 2, cudaMemcpyDeviceToDevice, s));
  rc = ops_.replay(s, use_graph_);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaMemcpyAsync(image, image_, img * 2, cudaMemcpyDeviceToDevice, s));
  return DLM_OK;
}

int VAEModel::decode_host(int B, int h, int w, const __half* latent, __half* image, cudaStream_t s) {
  DLM_REQUIRE(latent && image, DLM_ERR_INVALID, "vae_decode_host: null input");
  int rc = plan(B, h, w);
  if (rc != DLM_OK) return rc;
  const size_t lat = static_cast<size_t>(B) * kLatC * h * w;
  const size_t img = static_cast<size_t>(B) * 3 * 64 * h * w;
  DLM_CHECK_CUDA(cudaMemcpyAsync(lat_in_, latent, lat * 2, cudaMemcpyHostToDevice, s));
  rc = ops_.replay(s, use_graph_);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaMemcpyAsync(image, image_, img * 2, cudaMemcpyDeviceToHost, s));
  DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  return DLM_OK;
}

int VAEModel::time_ops(cudaStream_t s, double* ms, double* flops, int* count) {
  DLM_REQUIRE(abuf_ != nullptr, DLM_ERR_INVALID, "vae_time_ops: run a decode first");
  return ops_.time(s, ms, flops, count);
}

int VAEModel::stage(const std::string& name, const void** ptr, int* dtype, int* C, int* H,
                    int* Wd) const {
  auto it = stages_.find(name);
  DLM_REQUIRE(it != stages_.end(), DLM_ERR_NOT_FOUND, "vae: no stage %s", name.c_str());
  *ptr = it->second.ptr;
  *dtype = it->second.dtype;
  *C = it->second.C;
  *H = it->second.H;
  *Wd = it->second.W;
  return DLM_OK;
}

}  // namespace dlm

// ================================================================== C ABI

extern "C" {

int dlm_vae_create(int n, const char* const* names, const void* const* dev_ptrs,
                   const int64_t* numels, void** handle, void* stream) {
  DLM_REQUIRE(handle != nullptr && names != nullptr && dev_ptrs != nullptr && n > 0, DLM_ERR_INVALID,
              "vae_create: null argument");
  *handle = nullptr;
  auto* m = new (std::nothrow) dlm::VAEModel();
  DLM_REQUIRE(m != nullptr, DLM_ERR_NOMEM, "vae_create: out of host memory");
  int rc = m->create(n, names, dev_ptrs, numels, static_cast<cudaStream_t>(stream));
  if (rc != DLM_OK) {
    delete m;
    return rc;
  }
  *handle = m;
  return DLM_OK;
}

int dlm_vae_destroy(void* handle) {
  delete static_cast<dlm::VAEModel*>(handle);
  return DLM_OK;
}

int dlm_vae_decode(void* handle, int B, int h, int w, const void* latent, void* image, void* stream) {
  DLM_REQUIRE(handle != nullptr, DLM_ERR_INVALID, "vae_decode: null handle");
  return static_cast<dlm::VAEModel*>(handle)->decode(B, h, w, static_cast<const __half*>(latent),
                                                     static_cast<__half*>(image),
                                                     static_cast<cudaStream_t>(stream));
}

int dlm_vae_decode_host(void* handle, int B, int h, int w, const void* latent_host, void* image_host,
                        void* stream) {
  DLM_REQUIRE(handle != nullptr, DLM_ERR_INVALID, "vae_decode_host: null handle");
  return static_cast<dlm::VAEModel*>(handle)->decode_host(
      B, h, w, static_cast<const __half*>(latent_host), static_cast<__half*>(image_host),
      static_cast<cudaStream_t>(stream));
}

int dlm_vae_set_graph(void* handle, int enable) {
  DLM_REQUIRE(handle != nullptr, DLM_ERR_INVALID, "vae_set_graph: null handle");
  static_cast<dlm::VAEModel*>(handle)->set_graph(enable != 0);
  return DLM_OK;
}

int dlm_vae_stage(void* handle, const char* name, const void** ptr, int* dtype, int* C, int* H,
                  int* W) {
  DLM_REQUIRE(handle && name && ptr && dtype && C && H && W, DLM_ERR_INVALID,
              "vae_stage: null argument");
  return static_cast<const dlm::VAEModel*>(handle)->stage(name, ptr, dtype, C, H, W);
}

int dlm_vae_info(void* handle, int64_t* arena_bytes, int64_t* weight_bytes, int* num_launches) {
  DLM_REQUIRE(handle != nullptr, DLM_ERR_INVALID, "vae_info: null handle");
  const auto* m = static_cast<const dlm::VAEModel*>(handle);
  if (arena_bytes) *arena_bytes = static_cast<int64_t>(m->arena_bytes());
  if (weight_bytes) *weight_bytes = static_cast<int64_t>(m->weight_bytes());
  if (num_launches) *num_launches = m->num_launches();
  return DLM_OK;
}

int dlm_vae_time_ops(void* handle, double* ms, double* flops, int* count, void* stream) {
  DLM_REQUIRE(handle && ms && flops && count, DLM_ERR_INVALID, "vae_time_ops: null argument");
  return static_cast<dlm::VAEModel*>(handle)->time_ops(static_cast<cudaStream_t>(stream), ms, flops,
                                                       count);
}

int dlm_vae_weight_count(void) { return static_cast<int>(dlm::vae_weight_specs().size()); }

int dlm_vae_weight_info(int index, char* name, int name_cap, int64_t* shape, int* ndim) {
  DLM_REQUIRE(name && shape && ndim && name_cap > 0, DLM_ERR_INVALID, "vae_weight_info: null argument");
  const auto specs = dlm::vae_weight_specs();
  DLM_REQUIRE(index >= 0 && index < static_cast<int>(specs.size()), DLM_ERR_INVALID,
              "vae_weight_info: index %d out of range", index);
  const auto& sp = specs[index];
  DLM_REQUIRE(static_cast<int>(sp.name.size()) < name_cap, DLM_ERR_INVALID,
              "vae_weight_info: name buffer too small");
  std::memcpy(name, sp.name.c_str(), sp.name.size() + 1);
  *ndim = static_cast<int>(sp.shape.size());
  for (int i = 0; i < 4; ++i) shape[i] = i < *ndim ? sp.shape[i] : 0;
  return DLM_OK;
}

}  // extern "C"
