// Host-side common pieces (see common.h) and the library-level C-ABI entry points.
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.h"

namespace {

thread_local char g_last_error[1024] = "";

// Status word written by kernels that give up a bounded wait.  One per device (each device
// that loads the library holds its own copy of this variable).
__device__ int g_dlm_device_status = 0;

constexpr int kMaxDevices = 64;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

}  // namespace

namespace dlm {

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

bool pdl_enabled() {
  // Programmatic dependent launch is on by default (DLM_PDL=0 turns it off): every kernel that is
  // launched with it waits (griddepcontrol.wait) before its first global read or write, so only
  // its set-up (barriers, TMEM, descriptor prefetch) overlaps the previous kernel's tail.  The
  // UNet step measured 18.6 ms with it against 19.0 ms without (B200, graph replay).
  static const bool on = [] {
    const char* e = std::getenv("DLM_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int num_sms() {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int* device_status_ptr() {
  static int* cache[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dlm_device_status) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

bool encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (g_encode == nullptr) {
    set_error("cuTensorMapEncodeTiled entry point not available");
    return false;
  }
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  for (uint32_t i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
  }
  for (uint32_t i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d, rank %u)", static_cast<int>(r), rank);
    return false;
  }
  return true;
}

bool tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_rows, uint32_t box_cols) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t strides[1] = {ld * 2};
  const uint32_t box[2] = {box_cols, box_rows};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace dlm

extern "C" {

const char* dlm_last_error(void) { return g_last_error; }

const char* dlm_version(void) { return "dollama_b200 0.1 (sm_100a)"; }

int dlm_memcpy(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return DLM_OK;
  DLM_REQUIRE(dst != nullptr && src != nullptr, DLM_ERR_INVALID, "dlm_memcpy: null pointer");
  DLM_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
  return DLM_OK;
}

int dlm_get_device_status(int* out_code, int clear, void* stream) {
  DLM_REQUIRE(out_code != nullptr, DLM_ERR_INVALID, "dlm_get_device_status: null out_code");
  int* p = dlm::device_status_ptr();
  DLM_REQUIRE(p != nullptr, DLM_ERR_CUDA, "dlm_get_device_status: no device status symbol");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  DLM_CHECK_CUDA(cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, s));
  DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  if (clear && v != 0) {
    const int zero = 0;
    DLM_CHECK_CUDA(cudaMemcpyAsync(p, &zero, sizeof(int), cudaMemcpyHostToDevice, s));
    DLM_CHECK_CUDA(cudaStreamSynchronize(s));
  }
  *out_code = v;
  return DLM_OK;
}

}  // extern "C"
