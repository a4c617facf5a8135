// SDXL txt2img denoising loop on the device: Euler (epsilon) schedule, classifier-free guidance,
// UNet steps and the VAE decode, with no host round trip between steps.
//
// Replaces the loop of DiffusionPipeline::generate_txt2img (reference src/infer/diffusion.cu:
// 896-988), which per step copies the latent to the device, runs the UNet, copies both noise
// predictions back, combines them and takes the Euler step on the host (scheduler
// src/infer/scheduler.hpp).  Here the schedule is computed once on the host (the reference's
// EulerDiscreteScheduler restated: scaled_linear betas, "leading" spacing, steps_offset 1,
// np.interp of the training sigmas), and every step is three launches on one stream:
//   scale_latent_kernel  x_in = fp16(x / sqrt(sigma_i^2 + 1)) for both CFG halves
//                        (scale_model_input, scheduler.hpp:110-119)
//   UNet step            (CUDA graph, B = 2: cond, uncond)
//   cfg_euler_kernel     e = e_u + g (e_c - e_u) (diffusion.cu:972);
//                        x += e * (sigma_{i+1} - sigma_i) in double (scheduler.hpp:126-140)
// then the VAE input fp16(x / scaling_factor) (diffusion.cu:979-986) and the VAE decode.
#include <cmath>
#include <vector>

#include "common.h"
#include "unet.h"
#include "vae.h"

namespace dlm {

namespace {

// Euler schedule of the SDXL defaults (1000 training steps, scaled_linear betas 0.00085 ..
// 0.012, leading spacing, steps_offset 1): sigmas [steps + 1] (last 0), timesteps [steps].
void euler_schedule(int steps, std::vector<float>& sigmas, std::vector<float>& timesteps) {
  const int n_train = 1000;
  const double s0 = std::sqrt(0.00085), s1 = std::sqrt(0.012);
  std::vector<double> train(n_train);
  double cumprod = 1.0;
  for (int i = 0; i < n_train; ++i) {
    const double t = static_cast<double>(i) / (n_train - 1);
    const double sb = s0 + (s1 - s0) * t;
    cumprod *= 1.0 - sb * sb;
    train[i] = std::sqrt((1.0 - cumprod) / cumprod);
  }
  const int ratio = n_train / steps;
  sigmas.assign(steps + 1, 0.0f);
  timesteps.assign(steps, 0.0f);
  for (int i = 0; i < steps; ++i) {
    const int j = steps - 1 - i;  // descending
    const double t = std::round(static_cast<double>(j) * ratio) + 1.0;
    timesteps[i] = static_cast<float>(t);
    double sig;
    if (t <= 0.0) {
      sig = train.front();
    } else if (t >= n_train - 1) {
      sig = train.back();
    } else {
      const int lo = static_cast<int>(std::floor(t));
      const double frac = t - lo;
      sig = train[lo] + (train[lo + 1] - train[lo]) * frac;
    }
    sigmas[i] = static_cast<float>(sig);
  }
  sigmas[steps] = 0.0f;
}

__global__ void scale_latent_kernel(const float* __restrict__ x, __half* __restrict__ out2, int n,
                                    double scale) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const __half h = __float2half_rn(static_cast<float>(__dmul_rn(static_cast<double>(x[i]), scale)));
  out2[i] = h;      // cond half
  out2[n + i] = h;  // uncond half (same latent)
}

__global__ void cfg_euler_kernel(const __half* __restrict__ noise2, float* __restrict__ x, int n,
                                 float guidance, double dt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float ec = __half2float(noise2[i]), eu = __half2float(noise2[n + i]);
  const float e = __fadd_rn(eu, __fmul_rn(guidance, __fsub_rn(ec, eu)));
  x[i] = static_cast<float>(__dadd_rn(static_cast<double>(x[i]), __dmul_rn(static_cast<double>(e), dt)));
}

__global__ void vae_input_kernel(const float* __restrict__ x, __half* __restrict__ out, int n,
                                 float scaling) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float2half_rn(__fdiv_rn(x[i], scaling));
}

struct DenoiseBuffers {
  __half* lat2 = nullptr;    // [2, 4, H, W]
  __half* noise2 = nullptr;  // [2, 4, H, W]
  float* x = nullptr;        // [1, 4, H, W]
  __half* vae_in = nullptr;  // [1, 4, H, W]
  cudaStream_t s = nullptr;
  ~DenoiseBuffers() {
    if (lat2) cudaFreeAsync(lat2, s);
    if (noise2) cudaFreeAsync(noise2, s);
    if (x) cudaFreeAsync(x, s);
    if (vae_in) cudaFreeAsync(vae_in, s);
  }
};

int denoise(UNetModel* unet, int H, int W, const float* init, int steps, float guidance,
            const __half* ehs, const __half* te, const __half* tid, DenoiseBuffers& b,
            cudaStream_t s) {
  DLM_REQUIRE(unet && init && ehs && te && tid, DLM_ERR_INVALID, "sdxl_denoise: null argument");
  DLM_REQUIRE(steps > 0 && steps <= 1000, DLM_ERR_INVALID, "sdxl_denoise: steps %d", steps);
  const int n = 4 * H * W;
  b.s = s;
  DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&b.lat2), 2 * n * sizeof(__half), s));
  DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&b.noise2), 2 * n * sizeof(__half), s));
  DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&b.x), n * sizeof(float), s));
  DLM_CHECK_CUDA(cudaMemcpyAsync(b.x, init, n * sizeof(float), cudaMemcpyDefault, s));
  std::vector<float> sig, ts;
  euler_schedule(steps, sig, ts);
  const int blocks = (n + 255) / 256;
  for (int i = 0; i < steps; ++i) {
    const double sigma = sig[i];
    scale_latent_kernel<<<blocks, 256, 0, s>>>(b.x, b.lat2, n, 1.0 / std::sqrt(sigma * sigma + 1.0));
    DLM_CHECK_CUDA(cudaGetLastError());
    int rc = unet->forward(2, H, W, b.lat2, ts[i], ehs, te, tid, b.noise2, s);
    if (rc != DLM_OK) return rc;
    cfg_euler_kernel<<<blocks, 256, 0, s>>>(b.noise2, b.x, n, guidance,
                                            static_cast<double>(sig[i + 1]) - static_cast<double>(sig[i]));
    DLM_CHECK_CUDA(cudaGetLastError());
  }
  return DLM_OK;
}

}  // namespace

}  // namespace dlm

// ================================================================== C ABI

extern "C" {

int dlm_sdxl_schedule(int steps, float* sigmas, float* timesteps) {
  DLM_REQUIRE(steps > 0 && steps <= 1000 && sigmas && timesteps, DLM_ERR_INVALID,
              "sdxl_schedule: bad argument");
  std::vector<float> sig, ts;
  dlm::euler_schedule(steps, sig, ts);
  for (int i = 0; i <= steps; ++i) sigmas[i] = sig[i];
  for (int i = 0; i < steps; ++i) timesteps[i] = ts[i];
  return DLM_OK;
}

int dlm_sdxl_denoise(void* unet, int H, int W, const float* init_latent, int steps, float guidance,
                     const void* ehs, const void* text_embeds, const void* time_ids,
                     float* latent_out, void* stream) {
  DLM_REQUIRE(latent_out, DLM_ERR_INVALID, "sdxl_denoise: null output");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dlm::DenoiseBuffers b;
  int rc = dlm::denoise(static_cast<dlm::UNetModel*>(unet), H, W, init_latent, steps, guidance,
                        static_cast<const __half*>(ehs), static_cast<const __half*>(text_embeds),
                        static_cast<const __half*>(time_ids), b, s);
  if (rc != DLM_OK) return rc;
  DLM_CHECK_CUDA(cudaMemcpyAsync(latent_out, b.x, 4 * H * W * sizeof(float), cudaMemcpyDefault, s));
  return DLM_OK;
}

int dlm_sdxl_generate(void* unet, void* vae, int H, int W, const float* init_latent, int steps,
                      float guidance, const void* ehs, const void* text_embeds, const void* time_ids,
                      float vae_scaling, void* image, void* stream) {
  DLM_REQUIRE(vae && image && vae_scaling != 0.0f, DLM_ERR_INVALID, "sdxl_generate: bad argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dlm::DenoiseBuffers b;
  int rc = dlm::denoise(static_cast<dlm::UNetModel*>(unet), H, W, init_latent, steps, guidance,
                        static_cast<const __half*>(ehs), static_cast<const __half*>(text_embeds),
                        static_cast<const __half*>(time_ids), b, s);
  if (rc != DLM_OK) return rc;
  const int n = 4 * H * W;
  DLM_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&b.vae_in), n * sizeof(__half), s));
  dlm::vae_input_kernel<<<(n + 255) / 256, 256, 0, s>>>(b.x, b.vae_in, n, vae_scaling);
  DLM_CHECK_CUDA(cudaGetLastError());
  return static_cast<dlm::VAEModel*>(vae)->decode(1, H, W, b.vae_in, static_cast<__half*>(image), s);
}

}  // extern "C"
