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
