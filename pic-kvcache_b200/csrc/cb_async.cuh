// Asynchronous-copy primitives shared by the TMA kernels: shared-memory
// mbarriers with bounded waits, and the untiled bulk copies
// (cp.async.bulk) between global and shared memory.
//
// Every wait here gives up after kTimeoutNs of %globaltimer time; a caller
// that sees a failed wait records an error code in its device error word and
// returns instead of spinning forever.
#pragma once

#include <stdint.h>

namespace cb {
namespace async {

constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s: a wait that long is a bug

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity, called by all 32 lanes
// of a warp; the result is warp-uniform.  Lanes that already observed the
// phase keep polling it (a completed phase stays observable until the peer
// side can advance the barrier again, which requires this warp).  Gives up
// after kTimeoutNs measured by lane 0.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint64_t start = 0;
  const int lane = threadIdx.x & 31;
  for (uint32_t spin = 0;; ++spin) {
    const bool mine = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, mine)) return true;
    if ((spin & 255u) == 0) {
      int expired = 0;
      if (lane == 0) {
        const uint64_t now = global_ns();
        if (start == 0)
          start = now;
        else if (now - start > kTimeoutNs)
          expired = 1;
      }
      if (__shfl_sync(0xffffffffu, expired, 0)) return false;
    }
  }
}

// The same bounded wait for a single thread.
__device__ __forceinline__ bool mbar_wait_one(uint64_t* bar, uint32_t parity) {
  uint64_t start = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      const uint64_t now = global_ns();
      if (start == 0)
        start = now;
      else if (now - start > kTimeoutNs)
        return false;
    }
  }
}

// global -> shared, completion counted in bytes on `bar`.  Both addresses
// 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// shared -> global in the issuing thread's current bulk group.
__device__ __forceinline__ void bulk_store(void* dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// At most N of this thread's committed bulk groups may still be reading
// their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// bulk_wait_read with a run-time bound: exact for 0..15, larger bounds wait
// as for 15 (stricter than asked, never weaker).
__device__ __forceinline__ void bulk_wait_read_dyn(uint32_t n) {
  switch (n) {
#define CB_WAIT_READ_CASE(k) \
  case k:                    \
    bulk_wait_read<k>();     \
    break;
    CB_WAIT_READ_CASE(0) CB_WAIT_READ_CASE(1) CB_WAIT_READ_CASE(2) CB_WAIT_READ_CASE(3)
    CB_WAIT_READ_CASE(4) CB_WAIT_READ_CASE(5) CB_WAIT_READ_CASE(6) CB_WAIT_READ_CASE(7)
    CB_WAIT_READ_CASE(8) CB_WAIT_READ_CASE(9) CB_WAIT_READ_CASE(10) CB_WAIT_READ_CASE(11)
    CB_WAIT_READ_CASE(12) CB_WAIT_READ_CASE(13) CB_WAIT_READ_CASE(14) CB_WAIT_READ_CASE(15)
#undef CB_WAIT_READ_CASE
    default:
      bulk_wait_read<15>();  // deeper bounds only wait more than needed
      break;
  }
}

// At most N of this thread's committed bulk groups may still be in flight.
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Orders this thread's shared-memory accesses with later async-proxy
// (bulk copy) accesses to the same shared memory.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace async
}  // namespace cb
