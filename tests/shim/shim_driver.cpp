// Test driver of include/dollama_b200_shim.hpp: a C++ program that calls the B200 library only
// through the reference's own function names and types (namespace dollama, SafeTensors from the
// reference's src/io/safetensors.hpp, LoraModule from src/infer/lora.hpp), as the reference's
// Euler loop and kernel tests would once the shim replaces its kernel wrappers.
//
//   shim_driver unet DIR   DIR/unet.safetensors + lat/ehs/te/tid .bin (fp16, B = 2, 128x128)
//                          -> noise.bin; conv_in_weight.bin (unet_weight_device_ptr); with a
//                          LoRA on conv_in (lora_a / lora_b .bin): its weight, noise_lora.bin,
//                          and noise_clear.bin after unet_clear_loras
//   shim_driver vae DIR    DIR/vae.safetensors + lat.bin ([1,4,128,128]) -> image.bin, through
//                          the per-call launch_vae_decode(const SafeTensors&, ...)
//   shim_driver runner DIR the reference's diffusion-runner plugin (IDiffusionRunner, built by
//                          make_b200_diffusion_runner from DIR/unet.safetensors and
//                          DIR/vae.safetensors): run_txt2img(4 steps, seed 1234, cfg 7.5) on fp32
//                          cond / uncond embeddings from DIR -> rgb.bin (uint8 HWC) and the
//                          initial latent it drew (lat0.bin, fp32)
//   shim_driver ops DIR    NCHW launch_conv2d on a tensor-core shape and on a direct-path
//                          shape, launch_group_norm_silu, launch_group_norm in place,
//                          launch_attention; inputs / outputs as .bin files
// Exit status 0 on success; a std::runtime_error from the shim is printed and gives 1.
#include <cstdio>
#include <cstring>
#include <memory>
#include <fstream>
#include <string>
#include <vector>

#include "dollama_b200_runner.hpp"
#include "dollama_b200_shim.hpp"

namespace {

std::vector<uint16_t> read_bin(const std::string& path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) throw std::runtime_error("cannot read " + path);
  const size_t n = static_cast<size_t>(f.tellg());
  std::vector<uint16_t> v(n / 2);
  f.seekg(0);
  f.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n));
  return v;
}

void write_bin(const std::string& path, const void* p, size_t bytes) {
  std::ofstream f(path, std::ios::binary);
  f.write(static_cast<const char*>(p), static_cast<std::streamsize>(bytes));
}

struct Dev {
  __half* p = nullptr;
  size_t n = 0;
  explicit Dev(size_t elems) : n(elems) {
    if (cudaMalloc(reinterpret_cast<void**>(&p), elems * 2) != cudaSuccess) throw std::runtime_error("cudaMalloc");
  }
  explicit Dev(const std::vector<uint16_t>& h) : Dev(h.size()) {
    cudaMemcpy(p, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
  }
  ~Dev() { cudaFree(p); }
  void save(const std::string& path) const {
    std::vector<uint16_t> h(n);
    cudaMemcpy(h.data(), p, n * 2, cudaMemcpyDeviceToHost);
    write_bin(path, h.data(), n * 2);
  }
};

int run_unet(const std::string& d) {
  dollama::SafeTensors st(d + "/unet.safetensors");
  Dev lat(read_bin(d + "/lat.bin")), ehs(read_bin(d + "/ehs.bin")), te(read_bin(d + "/te.bin")),
      tid(read_bin(d + "/tid.bin"));
  Dev noise(lat.n);
  dollama::UnetWeightsHandle h = dollama::unet_weights_create(st);
  dollama::launch_unet_batched(h, 2, lat.p, 999.0f, ehs.p, te.p, tid.p, noise.p);
  noise.save(d + "/noise.bin");
  const __half* w = dollama::unet_weight_device_ptr(h, "conv_in.weight");
  std::vector<uint16_t> hw(320 * 4 * 9);
  cudaMemcpy(hw.data(), w, hw.size() * 2, cudaMemcpyDeviceToHost);
  write_bin(d + "/conv_in_weight.bin", hw.data(), hw.size() * 2);
  // a rank-4 LoRA on conv_in (A [4, 36], B [320, 4], scale 0.5): the weight as
  // unet_weight_device_ptr reports it, the step with it, and the step after clearing it
  dollama::LoraModule m;
  m.base_key = "conv_in.weight";
  m.a_fp16 = read_bin(d + "/lora_a.bin");
  m.b_fp16 = read_bin(d + "/lora_b.bin");
  m.rank = 4;
  m.in_flat = 36;
  m.out_dim = 320;
  m.scale = 0.5f;
  dollama::unet_apply_loras(h, &m, 1);
  w = dollama::unet_weight_device_ptr(h, "conv_in.weight");
  cudaMemcpy(hw.data(), w, hw.size() * 2, cudaMemcpyDeviceToHost);
  write_bin(d + "/conv_in_weight_lora.bin", hw.data(), hw.size() * 2);
  dollama::launch_unet_batched(h, 2, lat.p, 999.0f, ehs.p, te.p, tid.p, noise.p);
  noise.save(d + "/noise_lora.bin");
  dollama::unet_clear_loras(h);
  dollama::launch_unet_batched(h, 2, lat.p, 999.0f, ehs.p, te.p, tid.p, noise.p);
  noise.save(d + "/noise_clear.bin");
  dollama::unet_weights_destroy(h);
  return 0;
}

int run_vae(const std::string& d) {
  dollama::SafeTensors st(d + "/vae.safetensors");
  Dev lat(read_bin(d + "/lat.bin"));
  Dev img(size_t(3) * 1024 * 1024);
  dollama::launch_vae_decode(st, lat.p, img.p);
  img.save(d + "/image.bin");
  return 0;
}

std::vector<float> read_f32(const std::string& path) {
  std::vector<uint16_t> raw = read_bin(path);
  std::vector<float> v(raw.size() / 2);
  std::memcpy(v.data(), raw.data(), v.size() * 4);
  return v;
}

int run_runner(const std::string& d) {
  std::unique_ptr<dollama::IDiffusionRunner> r = dollama::make_b200_diffusion_runner(
      d + "/unet.safetensors", d + "/vae.safetensors", "", dollama::FastConfig{}, 0.13025f);
  if (!r) throw std::runtime_error("make_b200_diffusion_runner returned nullptr");
  const std::vector<float> ce = read_f32(d + "/cond_ehs.f32"), ct = read_f32(d + "/cond_te.f32"),
                           ue = read_f32(d + "/uncond_ehs.f32"), ut = read_f32(d + "/uncond_te.f32"),
                           tid = read_f32(d + "/tid.f32");
  std::vector<uint8_t> rgb;
  int w = 0, h = 0;
  r->run_txt2img(4, 1234, 7.5f, ce.data(), ct.data(), ue.data(), ut.data(), tid.data(), rgb, w, h);
  if (w != 1024 || h != 1024 || rgb.size() != static_cast<size_t>(w) * h * 3)
    throw std::runtime_error("run_txt2img: unexpected image size");
  write_bin(d + "/rgb.bin", rgb.data(), rgb.size());
  float sig[5], ts[4];
  if (dlm_sdxl_schedule(4, sig, ts) != DLM_OK) throw std::runtime_error("schedule");
  std::vector<float> lat(4 * 128 * 128);
  dollama::b200_initial_latent(1234, sig[0], lat.data(), lat.size());
  write_bin(d + "/lat0.bin", lat.data(), lat.size() * 4);
  // a factory that cannot load its weights returns nullptr (the reference's contract)
  if (dollama::make_b200_diffusion_runner(d + "/missing.safetensors", d + "/vae.safetensors", ""))
    throw std::runtime_error("factory did not return nullptr for missing weights");
  return 0;
}

int run_ops(const std::string& d) {
  {  // tensor-core shape: [2,64,32,32] * [128,64,3,3] stride 1 pad 1
    Dev x(read_bin(d + "/cx.bin")), w(read_bin(d + "/cw.bin")), b(read_bin(d + "/cb.bin"));
    Dev y(size_t(2) * 128 * 32 * 32);
    if (!dollama::conv2d_uses_gemm_bias_path(2, 64, 32, 32, 128, 3, 3, 1, 1, 1, 1, 1, 1))
      throw std::runtime_error("expected the tensor-core path");
    dollama::launch_conv2d(x.p, w.p, b.p, y.p, 2, 64, 32, 32, 128, 3, 3, 1, 1, 1, 1, 1, 1);
    y.save(d + "/conv_out.bin");
  }
  {  // direct shape: [1,3,17,19] * [5,3,3,3] stride 2 pad 1
    Dev x(read_bin(d + "/dx.bin")), w(read_bin(d + "/dw.bin")), b(read_bin(d + "/db.bin"));
    Dev y(size_t(5) * 9 * 10);
    if (dollama::conv2d_uses_gemm_bias_path(1, 3, 17, 19, 5, 3, 3, 2, 2, 1, 1, 1, 1))
      throw std::runtime_error("expected the direct path");
    dollama::launch_conv2d(x.p, w.p, b.p, y.p, 1, 3, 17, 19, 5, 3, 3, 2, 2, 1, 1, 1, 1);
    y.save(d + "/dconv_out.bin");
  }
  {  // GroupNorm + SiLU [2,320,16,16]; then plain GroupNorm in place on a copy
    Dev x(read_bin(d + "/gx.bin")), g(read_bin(d + "/gg.bin")), b(read_bin(d + "/gb.bin"));
    Dev y(x.n);
    dollama::launch_group_norm_silu(x.p, g.p, b.p, y.p, 2, 320, 16, 16, 32, 1e-5f);
    y.save(d + "/gn_silu_out.bin");
    dollama::launch_group_norm(x.p, g.p, b.p, x.p, 2, 320, 16, 16, 32, 1e-6f);
    x.save(d + "/gn_inplace_out.bin");
  }
  {  // attention [1, 2, 256, 64]
    Dev q(read_bin(d + "/aq.bin")), k(read_bin(d + "/ak.bin")), v(read_bin(d + "/av.bin"));
    Dev o(q.n);
    dollama::launch_attention(q.p, k.p, v.p, o.p, 1, 2, 256, 256, 64, 0.125f);
    o.save(d + "/attn_out.bin");
  }
  cudaDeviceSynchronize();
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: shim_driver {unet|vae|runner|ops} DIR\n");
    return 2;
  }
  const std::string cmd = argv[1], dir = argv[2];
  try {
    if (cmd == "unet") return run_unet(dir);
    if (cmd == "vae") return run_vae(dir);
    if (cmd == "ops") return run_ops(dir);
    if (cmd == "runner") return run_runner(dir);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "shim_driver %s: %s\n", cmd.c_str(), e.what());
    return 1;
  }
  std::fprintf(stderr, "unknown command %s\n", cmd.c_str());
  return 2;
}
