// Host-side common pieces: status codes, tensor-map encoding through the driver entry point,
// per-device properties and the device status word.
#pragma once

#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/dollama_b200.h"

namespace dlm {

// Number of SMs of the current device (cached per device).
int num_sms();

// Device address of this library's status word on the current device (kernels that give
// up a bounded wait record a nonzero code there).  Cached per device.
int* device_status_ptr();

// cuTensorMapEncodeTiled through cudaGetDriverEntryPoint (no link-time libcuda dependency).
// Returns false if the driver rejects the map.
bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Row-major fp16 matrix [rows, cols] with leading dimension `ld` (elements), box
// [box_rows, 64 cols], 128-byte swizzle.
bool tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows, uint32_t box_cols);

// Whether kernels are launched with programmatic dependent launch (default on; DLM_PDL=0 off).
bool pdl_enabled();

// Launches `kernel` with programmatic dependent launch when it is enabled: the kernel may start
// while the previous kernel in the stream finishes, so it must execute griddepcontrol.wait before
// its first global memory access.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Records the last host-side error message (thread-local), returned by dlm_last_error().
void set_error(const char* fmt, ...);

}  // namespace dlm

#define DLM_CHECK_CUDA(expr)                                                   \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess) {                                                   \
      ::dlm::set_error("%s:%d %s: %s", __FILE__, __LINE__, #expr,              \
                       cudaGetErrorString(_e));                                \
      return DLM_ERR_CUDA;                                                     \
    }                                                                          \
  } while (0)

#define DLM_REQUIRE(cond, code, ...)                                           \
  do {                                                                         \
    if (!(cond)) {                                                             \
      ::dlm::set_error(__VA_ARGS__);                                           \
      return (code);                                                           \
    }                                                                          \
  } while (0)
