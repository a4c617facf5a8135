// GroupNorm entry point for callers that cannot allocate device memory.
//
// dlm_group_norm_nhwc needs a caller-provided scratch buffer for its per-chunk partial sums.
// Some callers have no way to provide one: a host program whose device memory is owned and
// fully pre-reserved by its own arena (the reference reserves its UNet arena's live peak up
// front, src/kernels/device_arena.cuh:31-54, and hands out nothing else), or a loop that must not
// pay cudaMalloc's implicit device synchronisation between steps.  This variant keeps the
// partial sums in a fixed array in this library's device memory instead, so the call itself
// allocates nothing (no cudaMalloc / cudaFree / allocating library routine).
//
// Limits and sharing:
//   * the static array holds kNoAllocPartials float2 (256 KiB); dlm_group_norm_nhwc_noalloc rejects
//     problems whose partial sums would not fit (an error, nothing is launched);
//   * every GPU that loads the library holds its own copy of the array until the process exits;
//   * on a 148-SM B200 every image size fits for batches of up to 339 images (the partial-sum
//     count grows with the SM count and the batch, not with the image size beyond a few pixels);
//   * every call shares the array and leaves the last call's partial sums and statistics in it.
//     The array also holds the statistics pass's per-image arrival counters, whose position
//     depends on the batch N (they follow the N x 32 statistics slots), so a call cannot rely on
//     an earlier call having left them at zero: each call clears its own counters on its stream
//     (cudaMemsetAsync, which allocates nothing) before the statistics pass.  A call that failed
//     part-way leaves nothing behind for the next one for the same reason.  Calls whose work
//     overlaps on the GPU (different streams, or other threads) race on the array and give wrong
//     results — serialise them;
//   * the array's device address is looked up (cudaGetSymbolAddress) by the first call on each
//     device, with that device current; that first call should come before any stream capture.
#include <mutex>

#include "norm.h"

namespace {

constexpr size_t kNoAllocPartials = 32768;  // float2 entries: 256 KiB

static __device__ __align__(256) float2 g_gn_noalloc_partials[kNoAllocPartials];

constexpr int kMaxDev = 64;
float2* g_partials_addr[kMaxDev] = {nullptr};
std::mutex g_partials_mu;

// Device address of the static array on the current device (looked up once per device).
int partials_for_current_device(float2** out) {
  int dev = 0;
  DLM_CHECK_CUDA(cudaGetDevice(&dev));
  DLM_REQUIRE(dev >= 0 && dev < kMaxDev, DLM_ERR_UNSUPPORTED,
              "group_norm_nhwc_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_partials_mu);
  if (g_partials_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gn_noalloc_partials);
    DLM_REQUIRE(e == cudaSuccess && p != nullptr, DLM_ERR_CUDA,
                "group_norm_nhwc_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_partials_addr[dev] = static_cast<float2*>(p);
  }
  *out = g_partials_addr[dev];
  return DLM_OK;
}

}  // namespace

extern "C" {

size_t dlm_group_norm_nhwc_noalloc_capacity(void) { return kNoAllocPartials; }

int dlm_group_norm_nhwc_noalloc(const void* x1, int C1, const void* x2, int C2, int N, int HW,
                                const void* gamma, const void* beta, float eps, int groups,
                                int silu, void* out, void* stream) {
  if (N == 0 || HW == 0 || C1 + C2 == 0) return DLM_OK;
  DLM_REQUIRE(groups == 32, DLM_ERR_UNSUPPORTED, "group_norm_nhwc_noalloc: groups must be 32");
  float2* partials = nullptr;
  int rc = partials_for_current_device(&partials);
  if (rc != DLM_OK) return rc;
  dlm::GnOp op;
  rc = dlm::gn_plan(&op, static_cast<const __half*>(x1), C1, static_cast<const __half*>(x2), C2, N,
                    HW, static_cast<const __half*>(gamma), static_cast<const __half*>(beta), eps,
                    silu != 0, static_cast<__half*>(out), partials, kNoAllocPartials);
  if (rc == DLM_ERR_NOMEM) {
    dlm::set_error(
        "group_norm_nhwc_noalloc: batch N=%d needs more partial sums than the %zu-entry static "
        "scratch holds; use dlm_group_norm_nhwc with a caller scratch buffer",
        N, kNoAllocPartials);
    return DLM_ERR_INVALID;
  }
  if (rc != DLM_OK) return rc;
  // the counters sit after the N x 32 statistics slots, where an earlier call with another N may
  // have left statistics: zero them for this call on its own stream
  DLM_CHECK_CUDA(cudaMemsetAsync(op.counters, 0, dlm::gn_counter_bytes(N),
                                 static_cast<cudaStream_t>(stream)));
  return dlm::gn_launch(op, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
