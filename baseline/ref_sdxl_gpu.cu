// C entry points over the reference's OWN CUDA SDXL UNet and VAE decoder, unchanged and
// recompiled for sm_100a — the GPU comparator and the whole-model pin of the CPU oracle.
//
// This file is not part of the product: it is compiled (by baseline/build_ref_gpu.py) together
// with the reference's sources where they lie (src/infer/unet.cu, src/kernels/*.cu), and the
// resulting baseline/_ref_gpu/libref_sdxl_gpu.so is loaded only by the tests that pin the
// oracle's structure to the reference and by bench.py's comparator leg.  Nothing in
// dollama_b200/ loads it.
//
// The reference API it wraps (namespace dollama):
//   unet_weights_create(const SafeTensors&) / launch_unet_batched(handle, B, ...) /
//   unet_weights_destroy                         (src/infer/unet.cuh:90-146)
//   unet_set_stage_hook(UnetStageHook)           (src/infer/unet.cuh:53-54)
//   vae_weights_create / launch_vae_decode(handle, latent, image) / vae_weights_destroy
//                                                (src/kernels/vae_decode.cuh:66-75)
// The reference throws std::runtime_error on failure; every entry point here catches it and
// returns -1 with the message in ref_last_error().  Launches go to the default stream, as the
// reference's kernels do.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "infer/unet.cuh"
#include "kernels/vae_decode.cuh"

namespace {

std::string g_err;
std::map<std::string, std::vector<uint16_t>> g_stages;  // fp16 bit patterns per stage name

void capture_hook(const char* name, const __half* d_buf, size_t n) {
  std::vector<uint16_t>& v = g_stages[name];
  v.resize(n);
  cudaMemcpy(v.data(), d_buf, n * sizeof(uint16_t), cudaMemcpyDeviceToHost);
}

struct UNetRef {
  dollama::SafeTensors st;
  dollama::UnetWeightsHandle h = nullptr;
  explicit UNetRef(const char* path) : st(path) { h = dollama::unet_weights_create(st); }
  ~UNetRef() { dollama::unet_weights_destroy(h); }
};

struct VAERef {
  dollama::SafeTensors st;
  dollama::VaeWeightsHandle h = nullptr;
  explicit VAERef(const char* path) : st(path) { h = dollama::vae_weights_create(st); }
  ~VAERef() { dollama::vae_weights_destroy(h); }
};

template <typename F>
int guarded(F&& f) {
  try {
    f();
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      g_err = cudaGetErrorString(e);
      return -2;
    }
    return 0;
  } catch (const std::exception& ex) {
    g_err = ex.what();
    return -1;
  }
}

}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_err.c_str(); }

int ref_unet_open(const char* safetensors_path, void** out) {
  *out = nullptr;
  return guarded([&] { *out = new UNetRef(safetensors_path); });
}

void ref_unet_close(void* h) { delete static_cast<UNetRef*>(h); }

// latent [B,4,128,128], ehs [B,77,2048], text_embeds [B,1280], time_ids [6] -> noise [B,4,128,128],
// all fp16 device pointers; attn_fast / epilogue select the reference's FAST modes.
int ref_unet_forward(void* h, int B, const void* latent, float timestep, const void* ehs,
                     const void* text_embeds, const void* time_ids, void* noise_out, int attn_fast,
                     int epilogue) {
  return guarded([&] {
    dollama::launch_unet_batched(static_cast<UNetRef*>(h)->h, B,
                                 static_cast<const __half*>(latent), timestep,
                                 static_cast<const __half*>(ehs),
                                 static_cast<const __half*>(text_embeds),
                                 static_cast<const __half*>(time_ids),
                                 static_cast<__half*>(noise_out), attn_fast != 0, epilogue != 0);
  });
}

// Same launch with no synchronisation and no error check (for timing back-to-back steps with
// events on the default stream); returns -1 only when the reference throws.
int ref_unet_launch(void* h, int B, const void* latent, float timestep, const void* ehs,
                    const void* text_embeds, const void* time_ids, void* noise_out, int attn_fast,
                    int epilogue) {
  try {
    dollama::launch_unet_batched(static_cast<UNetRef*>(h)->h, B,
                                 static_cast<const __half*>(latent), timestep,
                                 static_cast<const __half*>(ehs),
                                 static_cast<const __half*>(text_embeds),
                                 static_cast<const __half*>(time_ids),
                                 static_cast<__half*>(noise_out), attn_fast != 0, epilogue != 0);
    return 0;
  } catch (const std::exception& ex) {
    g_err = ex.what();
    return -1;
  }
}

// Stage capture through the reference's golden-test hook (every dbg_stat point of launch_unet):
// on = 1 copies each stage output to host memory as the forward passes it, on = 0 removes the
// hook and drops the copies.
void ref_unet_capture_stages(int on) {
  g_stages.clear();
  dollama::unet_set_stage_hook(on ? capture_hook : nullptr);
}

// Copies the captured stage `name` (fp16, the reference's NCHW layout) into host_out (at most
// max_elems) and returns its element count; 0 when the stage was not captured.
size_t ref_unet_stage(const char* name, void* host_out, size_t max_elems) {
  auto it = g_stages.find(name);
  if (it == g_stages.end()) return 0;
  const size_t n = it->second.size() < max_elems ? it->second.size() : max_elems;
  if (host_out) std::memcpy(host_out, it->second.data(), n * sizeof(uint16_t));
  return it->second.size();
}

int ref_vae_open(const char* safetensors_path, void** out) {
  *out = nullptr;
  return guarded([&] { *out = new VAERef(safetensors_path); });
}

void ref_vae_close(void* h) { delete static_cast<VAERef*>(h); }

// latent [1,4,128,128] -> image [1,3,1024,1024], fp16 device pointers.
int ref_vae_decode(void* h, const void* latent, void* image) {
  return guarded([&] {
    dollama::launch_vae_decode(static_cast<VAERef*>(h)->h, static_cast<const __half*>(latent),
                               static_cast<__half*>(image));
  });
}

}  // extern "C"
