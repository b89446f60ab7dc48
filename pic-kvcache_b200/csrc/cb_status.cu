// Status strings and stream/context binding for the C ABI.
#include <stdarg.h>
#include <stdio.h>

#include <cuda.h>  // CUcontext / CUresult only; the driver is reached through the runtime

#include <map>
#include <mutex>
#include <utility>

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
    // A capturing stream rejects device queries: the capture is recorded on
    // the caller's current device, which must own the stream, so keep it.
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(reinterpret_cast<cudaStream_t>(stream), &capture);
    if (e != cudaSuccess) {
      set_error("cudaStreamIsCapturing failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
    if (capture != cudaStreamCaptureStatusNone) return CB_OK;
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

int current_context(void** context) {
  using GetCurrent = CUresult (*)(CUcontext*);
  static const GetCurrent get = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<GetCurrent>(fn);
  }();
  if (get == nullptr) {
    set_error("cuCtxGetCurrent is unavailable through the CUDA runtime");
    return CB_ERR_CUDA;
  }
  CUcontext ctx = nullptr;
  const CUresult r = get(&ctx);
  if (r != CUDA_SUCCESS || ctx == nullptr) {
    set_error("no current CUDA context on this thread (cuCtxGetCurrent: %d)", static_cast<int>(r));
    return CB_ERR_CUDA;
  }
  *context = ctx;
  return CB_OK;
}

int ensure_dynamic_smem(const void* func, size_t bytes) {
  // Keyed by context, not device ordinal: a context created after
  // cudaDeviceReset (or by another runtime) starts from the default limit.
  static std::mutex lock;
  static std::map<std::pair<void*, const void*>, size_t> granted;
  void* context = nullptr;
  const int rc = current_context(&context);
  if (rc != CB_OK) return rc;
  std::lock_guard<std::mutex> guard(lock);
  size_t& have = granted[std::make_pair(context, func)];
  if (bytes <= have) return CB_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(%zu bytes) failed: %s", bytes, cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  have = bytes;
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

extern "C" int cb_abi_version(void) { return 6; }

extern "C" const char* cb_last_error(void) { return cb::g_last_error; }

// Strided device -> host copy on the copy engine: `rows` rows of `row_bytes`,
// rows `src_pitch` apart in device memory and `dst_pitch` apart in (pinned)
// host memory.  One transfer for a Store batch whose chunks land in
// consecutive arena entries (row pitch = the entry size).
extern "C" int cb_copy_rows_d2h(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                                int64_t row_bytes, int64_t rows, void* stream) {
  using namespace cb;
  clear_error();
  CB_REQUIRE(rows >= 0 && row_bytes >= 0, "negative size");
  if (rows == 0 || row_bytes == 0) return CB_OK;
  CB_REQUIRE(dst != nullptr && src != nullptr, "null pointer argument");
  CB_REQUIRE(dst_pitch >= row_bytes && src_pitch >= row_bytes, "pitch smaller than a row");
  CB_BIND(stream, src);
  cudaError_t e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_pitch), src,
                                    static_cast<size_t>(src_pitch), static_cast<size_t>(row_bytes),
                                    static_cast<size_t>(rows), cudaMemcpyDeviceToHost,
                                    reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("cudaMemcpy2DAsync failed: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}
