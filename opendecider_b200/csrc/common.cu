// Error reporting, version and the device-side error word of libod_b200.
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace od {

static thread_local char g_err[1024] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = 0;
  return OD_OK;
}

// One error word per device, written by kernels whose bounded spin-waits give up (never by a trap).
__device__ int32_t g_device_error;

int32_t* device_error_word() {
  static int32_t* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int32_t*>(p);
  }
  return addr[dev];
}

}  // namespace od

extern "C" const char* od_last_error(void) { return od::g_err; }

extern "C" const char* od_version(void) { return "od_b200 0.1 sm_100a"; }

extern "C" int od_device_error(void* stream, int32_t* host_code) {
  OD_REQUIRE(host_code, "od_device_error: host_code is null");
  int32_t* w = od::device_error_word();
  if (!w) return od::fail(OD_ECUDA, "od_device_error: no device error word");
  cudaStream_t s = od::as_stream(stream);
  OD_CUDA_TRY(cudaMemcpyAsync(host_code, w, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  OD_CUDA_TRY(cudaStreamSynchronize(s));
  OD_CUDA_TRY(cudaMemsetAsync(w, 0, sizeof(int32_t), s));
  OD_CUDA_TRY(cudaStreamSynchronize(s));
  return od::ok();
}
