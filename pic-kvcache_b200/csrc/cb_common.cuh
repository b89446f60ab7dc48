// Shared helpers of the CacheBlend B200 kernels: status reporting, stream
// context binding, vector types and exact per-op rounding for bf16/fp16/fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cacheblend_b200.h"

namespace cb {

// Records a printf-style message as this thread's last error.
void set_error(const char* fmt, ...);
void clear_error();

// Makes the device that owns `stream` (or, for the legacy NULL stream, the
// device holding `device_ptr`) current on the calling thread, so launches
// land on the right device whatever device the caller's own CUDA runtime
// instance considers current.
int bind_stream(void* stream, const void* device_ptr);

// Converts the launch status into CB_OK / CB_ERR_CUDA.
int launch_status(const char* kernel);

// The CUDA context current on the calling thread (driver handle, fetched
// through the runtime's driver entry point; no driver link).  Per-context
// state -- a device symbol's address, a kernel's shared-memory attribute --
// is keyed by this handle: a device ordinal can name several contexts over a
// process's life (cudaDeviceReset, an FFI host with its own context).
int current_context(void** context);

// Raises `func`'s dynamic shared memory limit in the current context to at
// least `bytes`.  The attribute is only changed when a launch needs more than
// any earlier one, so steady-state calls (and calls inside a stream capture
// after a warm-up launch) make no attribute change.
int ensure_dynamic_smem(const void* func, size_t bytes);

constexpr int kSmCount = 148;  // B200: 2 dies x 74 SMs

// Largest power-of-two vector width (<= 16 bytes) that divides every value
// OR-ed into `acc` (addresses, strides, row sizes).
inline int vector_bytes(uint64_t acc) {
  if (acc == 0) return 16;
  int w = 1;
  while (w < 16 && (acc & (uint64_t)w) == 0) w <<= 1;
  return w;
}

template <int BYTES>
struct Vec;
template <>
struct Vec<16> {
  using T = uint4;
};
template <>
struct Vec<8> {
  using T = uint2;
};
template <>
struct Vec<4> {
  using T = uint32_t;
};
template <>
struct Vec<2> {
  using T = uint16_t;
};
template <>
struct Vec<1> {
  using T = uint8_t;
};

// Streaming (read-once) 16-byte load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
template <typename V>
__device__ __forceinline__ V ld_vec(const V* p) {
  return *p;
}
template <>
__device__ __forceinline__ uint4 ld_vec<uint4>(const uint4* p) {
  return ld_stream(p);
}

// ---- element types ---------------------------------------------------------
// to_f / round_to reproduce torch's elementwise semantics for reduced
// precision tensors: every op is evaluated in fp32 (correctly rounded) and the
// result rounded to nearest-even in the storage type.
template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// fp32 value of `v` rounded to T and widened back.
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

inline int dtype_bytes(int dtype) {
  switch (dtype) {
    case CB_DTYPE_BF16:
    case CB_DTYPE_FP16:
      return 2;
    case CB_DTYPE_FP32:
      return 4;
    default:
      return 0;
  }
}

}  // namespace cb

#define CB_REQUIRE(cond, ...)         \
  do {                                \
    if (!(cond)) {                    \
      ::cb::set_error(__VA_ARGS__);   \
      return CB_ERR_INVALID;          \
    }                                 \
  } while (0)

#define CB_SUPPORTED(cond, ...)       \
  do {                                \
    if (!(cond)) {                    \
      ::cb::set_error(__VA_ARGS__);   \
      return CB_ERR_UNSUPPORTED;      \
    }                                 \
  } while (0)

#define CB_BIND(stream, device_ptr)                         \
  do {                                                      \
    int _cb_rc = ::cb::bind_stream((stream), (device_ptr)); \
    if (_cb_rc != CB_OK) return _cb_rc;                     \
  } while (0)
