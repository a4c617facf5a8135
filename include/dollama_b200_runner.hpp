// dollama_b200_runner.hpp — the reference's diffusion-runner plugin on libdollama_b200.
//
// The reference's "sdxl" IDiffusionBackend (src/server/sdxl_backend.hpp) turns prompt / negative
// into cond / uncond embeddings with its text conditioner and hands them to an IDiffusionRunner
// (src/server/diffusion_runner.hpp:33-74) built by make_diffusion_runner.  B200DiffusionRunner
// is that runner on this library: the resident UNet / VAE handles of the shim
// (include/dollama_b200_shim.hpp), the whole CFG Euler loop and the VAE decode on the device in one
// call (dlm_sdxl_generate), and the reference's image convention (uint8 RGB, [y, x, c] row-major
// HWC, (x * 0.5 + 0.5) clamped to [0, 1], * 255, rounded).  A maintainer's diffusion_runner.cu
// defines
//
//     std::unique_ptr<IDiffusionRunner> make_diffusion_runner(const std::string& unet,
//         const std::string& vae, const std::string& embeds, const FastConfig& fast,
//         float vae_scaling) { return make_b200_diffusion_runner(unet, vae, embeds, fast, vae_scaling); }
//
// and the backend, the HTTP / CLI layers and the LoRA requests run unchanged.
//
// The initial latent is the reference's: randn(seed) * sigmas[0] from the same generator
// (src/infer/diffusion.cu:76-140: splitmix64-seeded xorshift128+ uniforms, Box-Muller pairs in
// double), so a seed means the same starting noise on both.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "dollama_b200_shim.hpp"
#include "server/diffusion_runner.hpp"

namespace dollama {

namespace b200_runner_detail {

// The reference's seeded standard-normal stream (same algorithm and constants, own code):
// splitmix64 seeds two xorshift128+ words; uniforms are the top 53 bits; Box-Muller in double
// yields pairs, the second kept for the next call; u1 below 1e-12 is redrawn.
class SeededNormal {
 public:
  explicit SeededNormal(uint64_t seed) : a_(mix(seed)), b_(mix(seed + 0x9E3779B97F4A7C15ULL)) {}
  double next() {
    if (spare_ok_) {
      spare_ok_ = false;
      return spare_;
    }
    double u1 = 0.0;
    do {
      u1 = uniform();
    } while (u1 <= 1e-12);
    const double u2 = uniform();
    const double radius = std::sqrt(-2.0 * std::log(u1));
    const double angle = 2.0 * 3.14159265358979323846 * u2;
    spare_ = radius * std::sin(angle);
    spare_ok_ = true;
    return radius * std::cos(angle);
  }

 private:
  static uint64_t mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
  }
  double uniform() {
    uint64_t s1 = a_;
    const uint64_t s0 = b_;
    a_ = s0;
    s1 ^= s1 << 23;
    b_ = s1 ^ s0 ^ (s1 >> 17) ^ (s0 >> 26);
    return static_cast<double>((b_ + s0) >> 11) * (1.0 / 9007199254740992.0);
  }
  uint64_t a_, b_;
  bool spare_ok_ = false;
  double spare_ = 0.0;
};

inline uint16_t f32_to_f16_bits(float f) {
  const __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

}  // namespace b200_runner_detail

// randn(seed) * sigma0 over n latent values, as the reference draws its initial latent.
inline void b200_initial_latent(uint64_t seed, float sigma0, float* out, size_t n) {
  b200_runner_detail::SeededNormal rng(seed);
  for (size_t i = 0; i < n; ++i) out[i] = static_cast<float>(rng.next() * static_cast<double>(sigma0));
}

// VAE image [3, H, W] fp16 (NCHW) -> uint8 RGB [H, W, 3], the reference's conversion.
inline void b200_image_to_rgb8(const std::vector<uint16_t>& img, int H, int W,
                               std::vector<uint8_t>& rgb) {
  rgb.assign(static_cast<size_t>(H) * W * 3, 0);
  for (int c = 0; c < 3; ++c)
    for (int y = 0; y < H; ++y)
      for (int x = 0; x < W; ++x) {
        __half_raw hr;
        hr.x = img[(static_cast<size_t>(c) * H + y) * W + x];
        float v = __half2float(__half(hr)) * 0.5f + 0.5f;
        v = v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
        const int q = static_cast<int>(v * 255.0f + 0.5f);
        rgb[(static_cast<size_t>(y) * W + x) * 3 + c] = static_cast<uint8_t>(q < 0 ? 0 : (q > 255 ? 255 : q));
      }
}

class B200DiffusionRunner : public IDiffusionRunner {
 public:
  static constexpr int kLatent = 128;  // 1024 x 1024 images, as the reference's runner

  B200DiffusionRunner(const std::string& unet_path, const std::string& vae_path, float vae_scaling)
      : unet_st_(unet_path), vae_st_(vae_path), vae_scaling_(vae_scaling) {
    unet_ = unet_weights_create(unet_st_);
    try {
      vae_ = vae_weights_create(vae_st_);
    } catch (...) {
      unet_weights_destroy(unet_);
      throw;
    }
  }
  ~B200DiffusionRunner() override {
    vae_weights_destroy(vae_);
    unet_weights_destroy(unet_);
  }
  B200DiffusionRunner(const B200DiffusionRunner&) = delete;
  B200DiffusionRunner& operator=(const B200DiffusionRunner&) = delete;

  // LoRA files (the reference's LoraFileRequest): loaded by the reference's own kohya loader
  // against the base UNet's SafeTensors and merged into the resident weights.
  void apply_loras(const std::vector<LoraFileRequest>& reqs) override {
    std::vector<LoraModule> mods;
    for (const LoraFileRequest& r : reqs) {
      SafeTensors lora(r.path);
      std::vector<LoraModule> m = load_lora_modules(unet_st_, lora, r.strength);
      mods.insert(mods.end(), m.begin(), m.end());
    }
    if (!mods.empty()) unet_apply_loras(unet_, mods.data(), static_cast<int>(mods.size()));
  }
  void clear_loras() override { unet_clear_loras(unet_); }

  void run_txt2img(int steps, uint64_t seed, float guidance, const float* cond_ehs,
                   const float* cond_te, const float* uncond_ehs, const float* uncond_te,
                   const float* time_ids, std::vector<uint8_t>& rgb_out, int& w, int& h) override {
    using namespace b200_runner_detail;
    constexpr size_t kEhs = 77 * 2048, kTe = 1280;
    const size_t nlat = static_cast<size_t>(4) * kLatent * kLatent;
    const size_t nimg = static_cast<size_t>(3) * 8 * kLatent * 8 * kLatent;
    std::vector<float> sig(static_cast<size_t>(steps) + 1), ts(static_cast<size_t>(steps));
    dlm_check(dlm_sdxl_schedule(steps, sig.data(), ts.data()), "run_txt2img");
    std::vector<float> lat(nlat);
    b200_initial_latent(seed, sig[0], lat.data(), nlat);
    // conditioning in the library's fp16 layout: batch 2, cond first
    std::vector<uint16_t> ehs(2 * kEhs), te(2 * kTe), tid(6);
    for (size_t i = 0; i < kEhs; ++i) {
      ehs[i] = f32_to_f16_bits(cond_ehs[i]);
      ehs[kEhs + i] = f32_to_f16_bits(uncond_ehs[i]);
    }
    for (size_t i = 0; i < kTe; ++i) {
      te[i] = f32_to_f16_bits(cond_te[i]);
      te[kTe + i] = f32_to_f16_bits(uncond_te[i]);
    }
    for (int i = 0; i < 6; ++i) tid[i] = f32_to_f16_bits(time_ids[i]);
    char* d = nullptr;
    const size_t bytes = nlat * 4 + (ehs.size() + te.size() + 8) * 2 + nimg * 2 + 4 * 256;
    if (cudaMalloc(reinterpret_cast<void**>(&d), bytes) != cudaSuccess)
      throw std::runtime_error("run_txt2img: cudaMalloc");
    auto up = [](size_t off) { return ((off + 255) / 256) * 256; };
    const size_t o_ehs = up(nlat * 4), o_te = up(o_ehs + ehs.size() * 2),
                 o_tid = up(o_te + te.size() * 2), o_img = up(o_tid + 16);
    float* d_lat = reinterpret_cast<float*>(d);
    char* d_ehs = d + o_ehs;
    char* d_te = d + o_te;
    char* d_tid = d + o_tid;
    char* d_img = d + o_img;
    int rc = DLM_OK;
    if (cudaMemcpy(d_lat, lat.data(), nlat * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_ehs, ehs.data(), ehs.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_te, te.data(), te.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(d_tid, tid.data(), tid.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
      rc = DLM_ERR_CUDA;
    if (rc == DLM_OK)
      rc = dlm_sdxl_generate(static_cast<shim_detail::UNetShim*>(unet_)->h, vae_, kLatent, kLatent,
                             d_lat, steps, guidance, d_ehs, d_te, d_tid, vae_scaling_, d_img,
                             nullptr);
    std::vector<uint16_t> img(nimg);
    if (rc == DLM_OK && cudaMemcpy(img.data(), d_img, nimg * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
      rc = DLM_ERR_CUDA;
    cudaFree(d);
    dlm_check(rc, "run_txt2img");
    w = h = 8 * kLatent;
    b200_image_to_rgb8(img, h, w, rgb_out);
  }

 private:
  SafeTensors unet_st_, vae_st_;
  UnetWeightsHandle unet_ = nullptr;
  VaeWeightsHandle vae_ = nullptr;
  float vae_scaling_;
};

// make_diffusion_runner's contract (diffusion_runner.hpp:82-86): nullptr when the weights cannot be
// loaded.  embeds_path (the reference's golden embeddings) and the FAST flags select nothing here.
inline std::unique_ptr<IDiffusionRunner> make_b200_diffusion_runner(
    const std::string& unet_weights, const std::string& vae_weights, const std::string& /*embeds*/,
    const FastConfig& /*fast_cfg*/ = FastConfig{},
    float vae_scaling_factor = kServerDefaultVaeScalingFactor) {
  try {
    return std::unique_ptr<IDiffusionRunner>(
        new B200DiffusionRunner(unet_weights, vae_weights, vae_scaling_factor));
  } catch (...) {
    return nullptr;
  }
}

}  // namespace dollama
