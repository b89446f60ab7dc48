// Status strings and stream/context binding for the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "cb_common.cuh"

namespace cb {

namespace {
thread_local char g_last_error[512] = {0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int bind_stream(void* stream, const void* device_ptr) {
  clear_error();
  int want = -1;
  cudaError_t e = cudaSuccess;
  if (stream != nullptr) {
    e = cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &want);
    if (e != cudaSuccess) {
      set_error("cudaStreamGetDevice failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
  } else if (device_ptr != nullptr) {
    // Legacy default stream: the output tensor's device decides.
    cudaPointerAttributes attr;
    e = cudaPointerGetAttributes(&attr, device_ptr);
    if (e != cudaSuccess) {
      set_error("cudaPointerGetAttributes failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
      set_error("output pointer is not device memory");
      return CB_ERR_INVALID;
    }
    want = attr.device;
  } else {
    return CB_OK;
  }
  int cur = -1;
  e = cudaGetDevice(&cur);
  if (e != cudaSuccess || cur != want) {
    e = cudaSetDevice(want);
    if (e != cudaSuccess) {
      set_error("cudaSetDevice(%d) failed: %s", want, cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
  }
  return CB_OK;
}

int launch_status(const char* kernel) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", kernel, cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

}  // namespace cb

extern "C" int cb_abi_version(void) { return 1; }

extern "C" const char* cb_last_error(void) { return cb::g_last_error; }
