// tcgen05 / TMA building blocks shared by the tensor-core kernels (Sparse-Q
// scorer, blend attention): shared-memory mbarriers with bounded waits, 3-D
// TMA tensor loads, K-major SWIZZLE_128B UMMA operand descriptors,
// tcgen05.mma / commit / fences, TMEM loads and stores, and the host-side
// tensor-map encoder fetched through the runtime (no driver link).
#pragma once

#include <cuda.h>  // CUtensorMap types; the encoder is fetched through the runtime

#include "cb_common.cuh"

namespace cb {
namespace tc {

constexpr int kTile = 128;                  // rows / keys / columns per operand tile
constexpr int kHalfBytes = kTile * 64 * 2;  // one 128x64 16-bit SW128 box
constexpr int kTileBytes = 2 * kHalfBytes;  // 32 KiB: a full 128x128 operand
constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s: a wait that long is a bug

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
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
// try_wait with a suspend-time hint: while the phase is incomplete the thread
// sleeps (up to hint_ns) until it completes instead of re-polling the barrier
// word.  Polling warps would otherwise compete for shared-memory bandwidth,
// which tcgen05.mma needs in full for its operands (a 128x128x16 product
// reads 8 KiB in 64 cycles).
constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms per try; the 2 s bound still applies
__device__ __forceinline__ bool mbar_try_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}
// Single-thread bounded wait (producer / MMA lanes).
__device__ __forceinline__ bool wait1(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (;;) {
    if (mbar_try_sleep(bar, parity)) return true;
    if (global_ns() - start > kTimeoutNs) return false;
  }
}
// Warp-uniform bounded wait (epilogue warps).  A lane that already observed
// the phase keeps observing it: the barrier cannot advance again before this
// warp arrives on its peer barrier.
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity) {
  if (__all_sync(0xffffffffu, mbar_try(bar, parity))) return true;
  const uint64_t start = global_ns();
  for (;;) {
    if (__all_sync(0xffffffffu, mbar_try_sleep(bar, parity))) return true;
    if (__shfl_sync(0xffffffffu, static_cast<int>(global_ns() - start > kTimeoutNs), 0)) return false;
  }
}
__device__ __forceinline__ void tma_load_4d(void* smem, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* smem, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// K-major, SWIZZLE_128B shared-memory matrix descriptor (sm_100 format):
// start>>4 | LBO(16 B)>>4 << 16 | SBO(1024 B = 8 rows x 128 B)>>4 << 32 |
// version 1 << 46 | layout SWIZZLE_128B (2) << 61, kept as two words: the high
// word is the same for every operand here (SBO 1024 B, version 1,
// SWIZZLE_128B), the low word holds the start address >> 4 (14 bits: shared
// memory stays below 256 KiB, so adding a K-step offset never carries into the
// LBO field).  Issuing an MMA then costs one add per operand instead of a
// 64-bit build.
constexpr uint32_t kDescHi = 64u | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t desc_lo(uint32_t smem_addr) {
  return ((smem_addr >> 4) & 0x3FFFu) | (1u << 16);
}
// Low-word offset of K step kk (16 elements = 32 B) within a 128x128 operand
// stored as two 128x64 SW128 halves 16 KiB apart.
__host__ __device__ constexpr uint32_t kstep_lo(int kk) {
  return static_cast<uint32_t>((kk >> 2) * (kHalfBytes >> 4) + (kk & 3) * 2);
}
// Eight K steps (K = 128) of a 128x128 product with both operands in shared
// memory, issued from one asm block: per step two adds and the MMA, nothing
// the issuing thread has to wait on, and only a few registers.
__device__ __forceinline__ void umma_k128(uint32_t tmem_d, uint32_t a_tile, uint32_t b_tile,
                                          uint32_t idesc, bool accumulate_first) {
  static_assert(kstep_lo(1) == 2 && kstep_lo(4) == 1024, "K-step offsets baked into umma_k128");
  asm volatile(
      "{\n\t.reg .b64 da, db;\n\t.reg .b32 a, b;\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 da, {%1, %5};\n\tmov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t"
      "add.u32 a, %1, 2;\n\tadd.u32 b, %2, 2;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 4;\n\tadd.u32 b, %2, 4;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 6;\n\tadd.u32 b, %2, 6;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1024;\n\tadd.u32 b, %2, 1024;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1026;\n\tadd.u32 b, %2, 1026;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1028;\n\tadd.u32 b, %2, 1028;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1030;\n\tadd.u32 b, %2, 1030;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t}" ::"r"(tmem_d),
      "r"(desc_lo(a_tile)), "r"(desc_lo(b_tile)), "r"(idesc), "r"(accumulate_first ? 1u : 0u),
      "n"(kDescHi));
}
// B operand stored MN-major (N contiguous), as a TMA tile of 128 K-rows x 64
// N-elements (SW128, 128 B per row) per box with the second 64 N-elements
// 16 KiB further: LBO = 16 KiB between the two N atoms, SBO = 1 KiB between
// 8-row K groups (the common high word), each K step of 16 rows 2 KiB further.
__device__ __forceinline__ uint32_t desc_lo_mn(uint32_t smem_addr) {
  return ((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint32_t>(kHalfBytes >> 4) << 16);
}
// Eight K steps (K = 128) with A K-major and B MN-major (instruction
// descriptor with the B-major bit set), both in shared memory.
__device__ __forceinline__ void umma_k128_bmn(uint32_t tmem_d, uint32_t a_tile, uint32_t b_tile,
                                              uint32_t idesc, bool accumulate_first) {
  static_assert(kstep_lo(1) == 2 && kstep_lo(4) == 1024, "K-step offsets baked into umma_k128_bmn");
  asm volatile(
      "{\n\t.reg .b64 da, db;\n\t.reg .b32 a, b;\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 da, {%1, %5};\n\tmov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t"
      "add.u32 a, %1, 2;\n\tadd.u32 b, %2, 128;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 4;\n\tadd.u32 b, %2, 256;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 6;\n\tadd.u32 b, %2, 384;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1024;\n\tadd.u32 b, %2, 512;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1026;\n\tadd.u32 b, %2, 640;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1028;\n\tadd.u32 b, %2, 768;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t"
      "add.u32 a, %1, 1030;\n\tadd.u32 b, %2, 896;\n\t"
      "mov.b64 da, {a, %5};\n\tmov.b64 db, {b, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, 1;\n\t}" ::"r"(tmem_d),
      "r"(desc_lo(a_tile)), "r"(desc_lo_mn(b_tile)), "r"(idesc), "r"(accumulate_first ? 1u : 0u),
      "n"(kDescHi));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 lanes x 32 consecutive fp32 columns of this warp's TMEM sub-partition.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 32 consecutive fp32 columns of this warp's TMEM sub-partition, stored.
__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31, %32};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline int get_encoder(EncodeTiled* fn) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr) {
    set_error("cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  *fn = reinterpret_cast<EncodeTiled>(ptr);
  return CB_OK;
}

// 3-D map with a 64 x b1 x b2 box of 16-bit elements, SWIZZLE_128B (inner box
// = 128 B), out-of-range elements read as zero.
inline int encode_3d(EncodeTiled encode, CUtensorMap* map, int dtype, const void* base, uint64_t d0,
              uint64_t d1, uint64_t d2, uint64_t stride1, uint64_t stride2, uint32_t b1,
              uint32_t b2) {
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1, stride2};
  const cuuint32_t box[3] = {64, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType type =
      dtype == CB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode(map, type, 3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return CB_ERR_INVALID;
  }
  return CB_OK;
}

// 4-D map with a 64 x b1 x b2 x b3 box of 16-bit elements, SWIZZLE_128B,
// out-of-range elements read as zero.
inline int encode_4d(EncodeTiled encode, CUtensorMap* map, int dtype, const void* base,
                     const uint64_t (&dims)[4], const uint64_t (&strides)[3], uint32_t b1,
                     uint32_t b2, uint32_t b3) {
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {strides[0], strides[1], strides[2]};
  const cuuint32_t box[4] = {64, b1, b2, b3};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType type =
      dtype == CB_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode(map, type, 4, const_cast<void*>(base), d, st, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (4-D) failed (%d)", static_cast<int>(r));
    return CB_ERR_INVALID;
  }
  return CB_OK;
}

}  // namespace tc
}  // namespace cb
