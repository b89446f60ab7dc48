// K2: fused per-layer blend load (APC prefix gather + gap zeroing + RoPE
// relocation + placement) and the standalone relocate_key kernel.
//
// Reference semantics: PagedBlendLoader.prefetch / _zero_gaps /
// _load_segments_fused / _load_segments_individually
// (cacheblend_vllm/ascend.py:224-370) and relocate_key (ascend.py:52-103).
// The staging row t of a layer is one of
//   * t < apc_prefix      -> paged gather of slot[t]            (ascend.py:233-247)
//   * gap                 -> zeros                              (ascend.py:280-287)
//   * hit of segment s    -> K relocated from source to target  (ascend.py:357)
//                            position, V copied; placed at t     (ascend.py:358-370)
// all written by one launch: one warp per (token, plane) row, 16-byte vectors.
// The hit source is any device-addressable memory: the device hit buffer
// filled by copy-engine H2D, or mapped pinned host memory (zero-copy load).
//
// Relocation arithmetic is bit-exact with torch's per-op evaluation in the
// key dtype: every product/sum is an fp32 op with round-to-nearest (explicit
// __fmul_rn/__fadd_rn/__fsub_rn, never contracted to FMA) followed by
// round-to-nearest-even back to the key dtype:
//   dc = r(r(nc*oc) + r(ns*os))     ds = r(r(ns*oc) - r(nc*os))
//   x1' = r(r(x1*dc) - r(x2*ds))    x2' = r(r(x2*dc) + r(x1*ds))
#include "cb_async.cuh"
#include "cb_common.cuh"

namespace cb {
namespace {

template <typename T, int N>
struct alignas(N * sizeof(T)) Pack {
  T v[N];
};

// VM: vector memory access (the caller guarantees N*sizeof(T) alignment);
// otherwise element by element, which only needs natural alignment.
template <typename T, int N, bool VM>
__device__ __forceinline__ Pack<T, N> load_pack(const T* p) {
  Pack<T, N> r;
  if constexpr (VM) {
    using V = typename Vec<N * sizeof(T)>::T;
    *reinterpret_cast<V*>(r.v) = *reinterpret_cast<const V*>(p);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) r.v[i] = p[i];
  }
  return r;
}

template <typename T, int N, bool VM>
__device__ __forceinline__ void store_pack(T* p, const Pack<T, N>& x) {
  if constexpr (VM) {
    using V = typename Vec<N * sizeof(T)>::T;
    *reinterpret_cast<V*>(p) = *reinterpret_cast<const V*>(x.v);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = x.v[i];
  }
}

template <typename T>
__device__ __forceinline__ void delta_rotation(float nc, float ns, float oc, float os, float& dc,
                                               float& ds) {
  dc = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(nc, oc)), rnd<T>(__fmul_rn(ns, os))));
  ds = rnd<T>(__fsub_rn(rnd<T>(__fmul_rn(ns, oc)), rnd<T>(__fmul_rn(nc, os))));
}

template <typename T>
__device__ __forceinline__ void rotate_pair(float a, float b, float dc, float ds, T& oa, T& ob) {
  oa = Elem<T>::from_f(__fsub_rn(rnd<T>(__fmul_rn(a, dc)), rnd<T>(__fmul_rn(b, ds))));
  ob = Elem<T>::from_f(__fadd_rn(rnd<T>(__fmul_rn(b, dc)), rnd<T>(__fmul_rn(a, ds))));
}

struct RopeDesc {
  const void* cos_sin;  // [max_position, rotary_dim], key dtype
  int64_t max_position;
  int rotary_dim;
  int head_size;
};

// ---- packed 2 x 16-bit arithmetic ------------------------------------------
// mul/add/sub.rn on bf16x2 / f16x2 round the exact result once to the 16-bit
// type.  That equals torch's evaluation (fp32 op, then round to the 16-bit
// type): a product of two 8-bit (bf16) or 11-bit (fp16) significands is exact
// in fp32, and a sum is either exact in fp32 or its smaller operand lies
// below half an ulp of the 16-bit result, where fp32 rounding cannot move the
// final rounding.  Explicit .rn keeps ptxas from contracting mul+add to fma.
template <typename T>
struct Packed;
template <>
struct Packed<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};
template <>
struct Packed<__half> {
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t add(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ uint32_t sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

// Delta rotation + rotation of one packed pair of lanes:
//   dc = nc*oc + ns*os, ds = ns*oc - nc*os, a' = a*dc - b*ds, b' = b*dc + a*ds
template <typename T>
__device__ __forceinline__ void packed_delta(uint32_t nc, uint32_t ns, uint32_t oc, uint32_t os,
                                             uint32_t& dc, uint32_t& ds) {
  using P = Packed<T>;
  dc = P::add(P::mul(nc, oc), P::mul(ns, os));
  ds = P::sub(P::mul(ns, oc), P::mul(nc, os));
}

// Relocates rotary item c (0 <= c < rotary items per head) of one head:
// NEOX pairs (i, i+half) for E consecutive i, or E/2 interleaved GPT-J pairs.
// Reads and writes only the item's own elements, so s == d (in place) is safe.
template <typename T, int E, bool NEOX, bool VM>
__device__ __forceinline__ void relocate_item(const T* s, T* d, int c, int rotary_dim,
                                              const T* old_cs, const T* new_cs) {
  const int R = rotary_dim;
  const int half = R / 2;
  constexpr bool kPacked = VM && sizeof(T) == 2;
  if constexpr (kPacked) {
    using P = Packed<T>;
    if constexpr (NEOX) {
      const int i0 = c * E;  // E == 8: four packed pairs of (i, i+1)
      const uint4 a = *reinterpret_cast<const uint4*>(s + i0);
      const uint4 b = *reinterpret_cast<const uint4*>(s + half + i0);
      const uint4 oc = *reinterpret_cast<const uint4*>(old_cs + i0);
      const uint4 os = *reinterpret_cast<const uint4*>(old_cs + half + i0);
      const uint4 nc = *reinterpret_cast<const uint4*>(new_cs + i0);
      const uint4 ns = *reinterpret_cast<const uint4*>(new_cs + half + i0);
      const uint32_t* A = &a.x;
      const uint32_t* B = &b.x;
      const uint32_t* OC = &oc.x;
      const uint32_t* OS = &os.x;
      const uint32_t* NC = &nc.x;
      const uint32_t* NS = &ns.x;
      uint4 ra, rb;
      uint32_t* RA = &ra.x;
      uint32_t* RB = &rb.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t dc, ds;
        packed_delta<T>(NC[k], NS[k], OC[k], OS[k], dc, ds);
        RA[k] = P::sub(P::mul(A[k], dc), P::mul(B[k], ds));
        RB[k] = P::add(P::mul(B[k], dc), P::mul(A[k], ds));
      }
      *reinterpret_cast<uint4*>(d + i0) = ra;
      *reinterpret_cast<uint4*>(d + half + i0) = rb;
    } else {
      const int i0 = c * E;  // 8 elements = pairs c*4 .. c*4+3
      const uint4 x = *reinterpret_cast<const uint4*>(s + i0);
      const uint2 oc = *reinterpret_cast<const uint2*>(old_cs + c * 4);
      const uint2 os = *reinterpret_cast<const uint2*>(old_cs + half + c * 4);
      const uint2 nc = *reinterpret_cast<const uint2*>(new_cs + c * 4);
      const uint2 ns = *reinterpret_cast<const uint2*>(new_cs + half + c * 4);
      uint32_t dc[2], ds[2];
      packed_delta<T>(nc.x, ns.x, oc.x, os.x, dc[0], ds[0]);
      packed_delta<T>(nc.y, ns.y, oc.y, os.y, dc[1], ds[1]);
      const uint32_t* X = &x.x;
      uint4 r;
      uint32_t* Rw = &r.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // broadcast pair k's (dc, ds) to both halves
        const uint32_t sel = (k & 1) ? 0x3232u : 0x1010u;
        const uint32_t dck = __byte_perm(dc[k >> 1], 0, sel);
        const uint32_t dsk = __byte_perm(ds[k >> 1], 0, sel);
        const uint32_t swapped = __byte_perm(X[k], 0, 0x1032u);      // (b, a)
        const uint32_t m1 = P::mul(X[k], dck);                        // (a*dc, b*dc)
        const uint32_t m2 = P::mul(swapped, dsk) ^ 0x00008000u;       // (-(b*ds), a*ds)
        Rw[k] = P::add(m1, m2);  // (a*dc - b*ds, b*dc + a*ds); x - y == x + (-y) exactly
      }
      *reinterpret_cast<uint4*>(d + i0) = r;
    }
  } else if constexpr (NEOX) {
    const int i0 = c * E;
    const Pack<T, E> a = load_pack<T, E, VM>(s + i0);
    const Pack<T, E> b = load_pack<T, E, VM>(s + half + i0);
    const Pack<T, E> oc = load_pack<T, E, VM>(old_cs + i0);
    const Pack<T, E> os = load_pack<T, E, VM>(old_cs + half + i0);
    const Pack<T, E> nc = load_pack<T, E, VM>(new_cs + i0);
    const Pack<T, E> ns = load_pack<T, E, VM>(new_cs + half + i0);
    Pack<T, E> ra, rb;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float dc, ds;
      delta_rotation<T>(Elem<T>::to_f(nc.v[e]), Elem<T>::to_f(ns.v[e]), Elem<T>::to_f(oc.v[e]),
                        Elem<T>::to_f(os.v[e]), dc, ds);
      rotate_pair<T>(Elem<T>::to_f(a.v[e]), Elem<T>::to_f(b.v[e]), dc, ds, ra.v[e], rb.v[e]);
    }
    store_pack<T, E, VM>(d + i0, ra);
    store_pack<T, E, VM>(d + half + i0, rb);
  } else {
    constexpr int P = E / 2;  // pairs per vector
    const int i0 = c * E;     // element offset; pair index c*P
    const Pack<T, E> x = load_pack<T, E, VM>(s + i0);
    const Pack<T, P> oc = load_pack<T, P, VM>(old_cs + c * P);
    const Pack<T, P> os = load_pack<T, P, VM>(old_cs + half + c * P);
    const Pack<T, P> nc = load_pack<T, P, VM>(new_cs + c * P);
    const Pack<T, P> ns = load_pack<T, P, VM>(new_cs + half + c * P);
    Pack<T, E> r;
#pragma unroll
    for (int e = 0; e < P; ++e) {
      float dc, ds;
      delta_rotation<T>(Elem<T>::to_f(nc.v[e]), Elem<T>::to_f(ns.v[e]), Elem<T>::to_f(oc.v[e]),
                        Elem<T>::to_f(os.v[e]), dc, ds);
      rotate_pair<T>(Elem<T>::to_f(x.v[2 * e]), Elem<T>::to_f(x.v[2 * e + 1]), dc, ds,
                     r.v[2 * e], r.v[2 * e + 1]);
    }
    store_pack<T, E, VM>(d + i0, r);
  }
}

// Relocates one token row (num_heads heads) with the whole warp.  old_cs /
// new_cs point at the rotary_dim-element cos|sin rows of the two positions.
// E = elements per work item: 16 bytes on the vector path (VM), 1 (neox) or
// 2 (one GPT-J pair) on the element-wise path.  16-bit types on the vector
// path use packed arithmetic, everything else per-element fp32 ops + rounding.
template <typename T, int E, bool NEOX, bool VM>
__device__ void warp_relocate_row(const T* src, int64_t src_hs, T* dst, int64_t dst_hs,
                                  int num_heads, int head_size, int rotary_dim, const T* old_cs,
                                  const T* new_cs, int lane) {
  const int R = rotary_dim;
  const int D = head_size;
  const int half = R / 2;
  // rotary items per head: neox pairs (i, i+half) in groups of E; GPT-J
  // interleaved pairs in vectors of E elements (E/2 pairs).
  const int rot_items = NEOX ? half / E : R / E;
  const int pass_items = (D - R) / E;
  const int per_head = rot_items + pass_items;
  const int items = num_heads * per_head;
  for (int it = lane; it < items; it += 32) {
    const int h = it / per_head;
    const int c = it - h * per_head;
    const T* s = src + h * src_hs;
    T* d = dst + h * dst_hs;
    if (c >= rot_items) {
      const int off = R + (c - rot_items) * E;
      store_pack<T, E, VM>(d + off, load_pack<T, E, VM>(s + off));
      continue;
    }
    relocate_item<T, E, NEOX, VM>(s, d, c, rotary_dim, old_cs, new_cs);
  }
}

// Table rows of a position (cos half then sin half).
template <typename T>
__device__ __forceinline__ const T* rope_row(const RopeDesc& rope, int64_t pos) {
  return static_cast<const T*>(rope.cos_sin) + pos * rope.rotary_dim;
}

// Plain warp row copy with VB-byte vectors.  GSRC: the source is global
// memory read once (non-coherent streaming loads); otherwise a generic load
// (shared-memory staging).
template <int VB, bool GSRC = true>
__device__ __forceinline__ void warp_copy_heads(const char* src, int64_t src_hs, char* dst,
                                                int64_t dst_hs, int num_heads, int units_per_head,
                                                int lane) {
  using V = typename Vec<VB>::T;
  constexpr int U = 4;
  const int units = num_heads * units_per_head;
  for (int i0 = lane; i0 < units; i0 += 32 * U) {
    V tmp[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * 32;
      if (i < units) {
        const int h = i / units_per_head;
        const int j = i - h * units_per_head;
        const V* p = reinterpret_cast<const V*>(src + h * src_hs + (int64_t)j * VB);
        if constexpr (GSRC)
          tmp[u] = ld_vec(p);
        else
          tmp[u] = *p;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * 32;
      if (i < units) {
        const int h = i / units_per_head;
        const int j = i - h * units_per_head;
        *reinterpret_cast<V*>(dst + h * dst_hs + (int64_t)j * VB) = tmp[u];
      }
    }
  }
}

template <int VB>
__device__ __forceinline__ void warp_zero_heads(char* dst, int64_t dst_hs, int num_heads,
                                                int units_per_head, int lane) {
  using V = typename Vec<VB>::T;
  const int units = num_heads * units_per_head;
  V z;
  memset(&z, 0, sizeof(V));
  for (int i = lane; i < units; i += 32) {
    const int h = i / units_per_head;
    const int j = i - h * units_per_head;
    *reinterpret_cast<V*>(dst + h * dst_hs + (int64_t)j * VB) = z;
  }
}

struct LoadArgs {
  char* out;
  int64_t out_plane_stride;
  int64_t out_token_stride;
  int64_t out_head_stride;
  int64_t alloc_end;
  int64_t apc_prefix;
  const char* k_cache;
  const char* v_cache;
  int64_t block_stride;
  int64_t slot_stride;
  int64_t head_stride;
  int64_t num_slots;
  uint32_t block_size;
  const int64_t* slots;
  int num_heads;
  const int32_t* token_segment;
  const cb_segment_t* segments;
  int64_t num_segments;
  RopeDesc rope;
};

template <typename T, int E, bool NEOX>
__global__ void __launch_bounds__(256) blend_load_kernel(LoadArgs a) {
  // 16-byte vectors on the vector path, single elements otherwise
  constexpr bool VM = E * sizeof(T) == 16;
  constexpr int VB = VM ? 16 : sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t tasks = 2 * a.alloc_end;
  const int units = a.rope.head_size * static_cast<int>(sizeof(T)) / VB;
  for (int64_t task = warp; task < tasks; task += nwarps) {
    const int64_t t = task >> 1;
    const int plane = static_cast<int>(task & 1);
    char* dst = a.out + plane * a.out_plane_stride + t * a.out_token_stride;
    if (t < a.apc_prefix) {
      int64_t s = __ldg(a.slots + t);
      if (s < 0) s += a.num_slots;
      if (s < 0 || s >= a.num_slots) continue;
      const uint32_t us = static_cast<uint32_t>(s);
      const uint32_t blk = us / a.block_size;
      const uint32_t off = us - blk * a.block_size;
      const char* src = (plane ? a.v_cache : a.k_cache) + (int64_t)blk * a.block_stride +
                        (int64_t)off * a.slot_stride;
      warp_copy_heads<VB>(src, a.head_stride, dst, a.out_head_stride, a.num_heads, units, lane);
      continue;
    }
    const int32_t seg_id = __ldg(a.token_segment + t);
    if (seg_id < 0 || seg_id >= a.num_segments) {
      warp_zero_heads<VB>(dst, a.out_head_stride, a.num_heads, units, lane);
      continue;
    }
    const cb_segment_t seg = a.segments[seg_id];
    const int64_t rel = t - seg.target_start;
    const int64_t old_pos = seg.source_start + rel;
    const bool rotate = plane == 0 && seg.rotate;
    if (rel < 0 || rel >= seg.length ||
        (rotate && (old_pos < 0 || old_pos >= a.rope.max_position || t >= a.rope.max_position))) {
      // Inconsistent descriptor (rejected by host validation): never read
      // outside the segment or the cos/sin table.
      warp_zero_heads<VB>(dst, a.out_head_stride, a.num_heads, units, lane);
      continue;
    }
    const char* src = reinterpret_cast<const char*>(plane ? seg.v_src : seg.k_src) +
                      rel * seg.src_token_stride;
    // Sources may be arbitrary device-addressable memory: take the scalar
    // path for a row whose source is not aligned to the vector width.
    const bool aligned = ((reinterpret_cast<uint64_t>(src) | (uint64_t)seg.src_head_stride) &
                          (uint64_t)(VB - 1)) == 0;
    if (((reinterpret_cast<uint64_t>(src) | (uint64_t)seg.src_head_stride) & (sizeof(T) - 1)) != 0) {
      warp_zero_heads<VB>(dst, a.out_head_stride, a.num_heads, units, lane);  // not even
      continue;                                                               // element-aligned
    }
    const int64_t src_hs = seg.src_head_stride / (int64_t)sizeof(T);
    const int64_t dst_hs = a.out_head_stride / (int64_t)sizeof(T);
    if (rotate) {
      const T* ocs = rope_row<T>(a.rope, old_pos);
      const T* ncs = rope_row<T>(a.rope, t);
      if (aligned)
        warp_relocate_row<T, E, NEOX, VM>(reinterpret_cast<const T*>(src), src_hs,
                                          reinterpret_cast<T*>(dst), dst_hs, a.num_heads,
                                          a.rope.head_size, a.rope.rotary_dim, ocs, ncs, lane);
      else
        warp_relocate_row<T, NEOX ? 1 : 2, NEOX, false>(
            reinterpret_cast<const T*>(src), src_hs, reinterpret_cast<T*>(dst), dst_hs,
            a.num_heads, a.rope.head_size, a.rope.rotary_dim, ocs, ncs, lane);
    } else if (aligned) {
      warp_copy_heads<VB>(src, seg.src_head_stride, dst, a.out_head_stride, a.num_heads, units,
                          lane);
    } else {
      warp_copy_heads<sizeof(T)>(src, seg.src_head_stride, dst, a.out_head_stride, a.num_heads,
                                 a.rope.head_size, lane);
    }
  }
}

// ---------------------------------------------------------------------------
// TMA-staged variant: a producer warp moves whole token rows (or per-head
// pieces) HBM -> shared memory with cp.async.bulk into a kStages-deep ring of
// 16 KiB tiles guarded by mbarriers; eight consumer warps relocate K / copy V
// out of shared memory into the staging buffer with 16-byte stores.  Bytes in
// flight cost no registers (up to 3 CTAs x 64 KiB per SM), which is what an
// HBM-bound gather with dependent address computation needs.  Used when every
// address is 16-byte aligned and the sources are device memory.
namespace tma {
constexpr int kStages = 3;
constexpr int kConsumerWarps = 8;
constexpr int kThreads = 32 * (1 + kConsumerWarps);
constexpr int kTileBytes = 20480;  // 8 rows of 8 bf16 heads x 128 + their cos|sin rows
constexpr int kMaxRows = 64;
using namespace ::cb::async;

enum : int32_t {
  kNone = 0,          // past alloc_end
  kSmemCopy = 1,      // staged by TMA, copied out
  kSmemRotate = 2,    // staged by TMA, relocated out
  kZero = 3,          // gap (or an inconsistent descriptor): zeros
  kDirectCopy = 4,    // source not 16-byte aligned: element-wise global copy
  kDirectRotate = 5,  // same, relocated
};

struct RowMeta {
  int64_t src;
  int64_t src_hs;
  int32_t kind;
  int32_t old_pos;
};

constexpr int kSmemSegments = 256;  // segment tables up to this size are copied to smem
constexpr size_t kFixedSmemBytes = kStages * kTileBytes + kStages * kMaxRows * sizeof(RowMeta) +
                                   2 * kStages * sizeof(uint64_t);
// dynamic shared memory of a launch: ring + row metadata + barriers + the
// segment table when it is small enough to live in shared memory
inline size_t smem_bytes(int64_t num_segments) {
  return kFixedSmemBytes +
         (num_segments <= kSmemSegments ? num_segments * sizeof(cb_segment_t) : 0);
}

__device__ __forceinline__ void report(int32_t* error, int32_t code) {
  if (error != nullptr) atomicCAS(error, 0, code);
}

// Raw per-row inputs the producer prefetches one tile ahead: the slot of an
// APC-prefix row, or the segment index of any other row.
struct RowRaw {
  int64_t slot;
  int32_t seg;
};

__device__ __forceinline__ RowRaw load_raw(const LoadArgs& a, int64_t t) {
  RowRaw raw{-1, -1};
  if (t >= a.alloc_end) return raw;
  if (t < a.apc_prefix)
    raw.slot = __ldg(a.slots + t);
  else
    raw.seg = __ldg(a.token_segment + t);
  return raw;
}

// Classifies one staging row (producer side); `segs` is the segment table in
// shared memory when it fits there, else in global memory.
__device__ RowMeta classify_row(const LoadArgs& a, const cb_segment_t* segs, int plane, int64_t t,
                                const RowRaw& raw, int head_bytes, int esize) {
  RowMeta m{0, 0, kNone, 0};
  if (t >= a.alloc_end) return m;
  m.kind = kZero;
  int64_t src;
  int64_t src_hs;
  bool rotate = false;
  if (t < a.apc_prefix) {
    int64_t slot = raw.slot;
    if (slot < 0) slot += a.num_slots;
    if (slot < 0 || slot >= a.num_slots) return m;
    const uint32_t us = static_cast<uint32_t>(slot);
    const uint32_t blk = us / a.block_size;
    const uint32_t off = us - blk * a.block_size;
    src = reinterpret_cast<int64_t>(plane ? a.v_cache : a.k_cache) + (int64_t)blk * a.block_stride +
          (int64_t)off * a.slot_stride;
    src_hs = a.head_stride;
  } else {
    const int32_t seg_id = raw.seg;
    if (seg_id < 0 || seg_id >= a.num_segments) return m;
    const cb_segment_t seg = segs[seg_id];
    const int64_t rel = t - seg.target_start;
    rotate = plane == 0 && seg.rotate;
    m.old_pos = static_cast<int32_t>(seg.source_start + rel);
    if (rel < 0 || rel >= seg.length) return m;
    if (rotate && (seg.source_start + rel < 0 || seg.source_start + rel >= a.rope.max_position ||
                   t >= a.rope.max_position))
      return m;
    src = static_cast<int64_t>(plane ? seg.v_src : seg.k_src) + rel * seg.src_token_stride;
    src_hs = seg.src_head_stride;
  }
  const uint64_t addr_bits = static_cast<uint64_t>(src) | static_cast<uint64_t>(src_hs);
  if (addr_bits & static_cast<uint64_t>(esize - 1)) return m;  // not even element-aligned: zeros
  m.src = src;
  m.src_hs = src_hs;
  if ((addr_bits & 15u) == 0 && (head_bytes & 15) == 0)
    m.kind = rotate ? kSmemRotate : kSmemCopy;
  else
    m.kind = rotate ? kDirectRotate : kDirectCopy;
  return m;
}

template <typename T, bool NEOX>
__global__ void __launch_bounds__(kThreads, 3) blend_load_tma_kernel(LoadArgs a, int rows_per_tile,
                                                                   int64_t tiles, int32_t* error) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + kStages * kTileBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + kStages * kMaxRows);
  uint64_t* empty = full + kStages;
  cb_segment_t* seg_smem = reinterpret_cast<cb_segment_t*>(empty + kStages);
  constexpr int E = 16 / sizeof(T);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head_bytes = a.rope.head_size * static_cast<int>(sizeof(T));
  const int row_bytes = a.num_heads * head_bytes;
  // per stage: rows_per_tile data rows, then one cos|sin row pair per data row
  const int cs_row_bytes = a.rope.rotary_dim * static_cast<int>(sizeof(T));
  const int cs_offset = rows_per_tile * row_bytes;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const bool segs_in_smem = a.num_segments <= kSmemSegments;
  if (segs_in_smem) {
    // 8-byte words: cb_segment_t's own alignment, whatever the caller's pointer
    const int words = static_cast<int>(a.num_segments * sizeof(cb_segment_t) / sizeof(uint2));
    const uint2* from = reinterpret_cast<const uint2*>(a.segments);
    uint2* to = reinterpret_cast<uint2*>(seg_smem);
    for (int i = threadIdx.x; i < words; i += blockDim.x) to[i] = from[i];
  }
  __syncthreads();
  const cb_segment_t* segs = segs_in_smem ? seg_smem : a.segments;

  if (warp == 0) {
    // ---- producer: classify the tile's rows, then stage them with TMA.  The
    // raw per-row indices of the next tile are loaded before waiting for a
    // free stage, so their latency hides behind the ring.
    RowRaw raw[2], raw_next[2];
    {
      const int64_t tok0 = (static_cast<int64_t>(blockIdx.x) >> 1) * rows_per_tile;
      raw[0] = load_raw(a, blockIdx.x < tiles && lane < rows_per_tile ? tok0 + lane : a.alloc_end);
      raw[1] = load_raw(a, blockIdx.x < tiles && lane + 32 < rows_per_tile ? tok0 + lane + 32
                                                                             : a.alloc_end);
    }
    int j = 0;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
      const int st = j % kStages;
      const uint32_t phase = (j / kStages) & 1u;
      const int64_t next = tile + gridDim.x;
      const int64_t next0 = (next >> 1) * rows_per_tile;
      raw_next[0] = load_raw(a, next < tiles && lane < rows_per_tile ? next0 + lane : a.alloc_end);
      raw_next[1] = load_raw(a, next < tiles && lane + 32 < rows_per_tile ? next0 + lane + 32
                                                                           : a.alloc_end);
      if (!mbar_wait(&empty[st], phase ^ 1u)) {
        if (lane == 0) report(error, 1);
        return;
      }
      const int plane = static_cast<int>(tile & 1);
      const int64_t tok0 = (tile >> 1) * rows_per_tile;
      uint32_t bytes = 0;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int r = lane + 32 * q;
        if (r >= rows_per_tile) continue;
        const RowMeta m = classify_row(a, segs, plane, tok0 + r, raw[q], head_bytes, sizeof(T));
        meta[st * kMaxRows + r] = m;
        if (m.kind == kSmemCopy) bytes += row_bytes;
        if (m.kind == kSmemRotate) bytes += row_bytes + 2 * cs_row_bytes;
      }
      raw[0] = raw_next[0];
      raw[1] = raw_next[1];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
      __syncwarp();
      if (lane == 0) {
        if (bytes)
          mbar_arrive_expect_tx(&full[st], bytes);
        else
          mbar_arrive(&full[st]);
      }
      __syncwarp();
      for (int r = lane; r < rows_per_tile; r += 32) {
        const RowMeta m = meta[st * kMaxRows + r];
        if (m.kind != kSmemCopy && m.kind != kSmemRotate) continue;
        unsigned char* dst = ring + st * kTileBytes + r * row_bytes;
        if (m.src_hs == head_bytes) {
          bulk_load(dst, reinterpret_cast<const void*>(m.src), row_bytes, &full[st]);
        } else {
          for (int h = 0; h < a.num_heads; ++h)
            bulk_load(dst + h * head_bytes, reinterpret_cast<const void*>(m.src + h * m.src_hs),
                      head_bytes, &full[st]);
        }
        if (m.kind == kSmemRotate) {
          unsigned char* cs = ring + st * kTileBytes + cs_offset + r * 2 * cs_row_bytes;
          bulk_load(cs, rope_row<T>(a.rope, m.old_pos), cs_row_bytes, &full[st]);
          bulk_load(cs + cs_row_bytes, rope_row<T>(a.rope, tok0 + r), cs_row_bytes, &full[st]);
        }
      }
    }
    return;
  }

  // ---- consumers
  const int cw = warp - 1;
  const int units = head_bytes / 16;
  int j = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
    const int st = j % kStages;
    const uint32_t phase = (j / kStages) & 1u;
    if (!mbar_wait(&full[st], phase)) {
      if (lane == 0) report(error, 2);
      return;
    }
    const int plane = static_cast<int>(tile & 1);
    const int64_t tok0 = (tile >> 1) * rows_per_tile;
    for (int r = cw; r < rows_per_tile; r += kConsumerWarps) {
      const RowMeta m = meta[st * kMaxRows + r];
      if (m.kind == kNone) continue;
      const int64_t t = tok0 + r;
      char* dst = a.out + plane * a.out_plane_stride + t * a.out_token_stride;
      const char* staged = reinterpret_cast<const char*>(ring + st * kTileBytes + r * row_bytes);
      const int64_t dst_hs = a.out_head_stride / (int64_t)sizeof(T);
      switch (m.kind) {
        case kSmemCopy:
          warp_copy_heads<16, false>(staged, head_bytes, dst, a.out_head_stride, a.num_heads, units,
                                     lane);
          break;
        case kSmemRotate: {
          const T* cs = reinterpret_cast<const T*>(ring + st * kTileBytes + cs_offset +
                                                   r * 2 * cs_row_bytes);
          warp_relocate_row<T, E, NEOX, true>(reinterpret_cast<const T*>(staged),
                                              a.rope.head_size, reinterpret_cast<T*>(dst), dst_hs,
                                              a.num_heads, a.rope.head_size, a.rope.rotary_dim,
                                              cs, cs + a.rope.rotary_dim, lane);
          break;
        }
        case kDirectCopy:
          warp_copy_heads<sizeof(T)>(reinterpret_cast<const char*>(m.src), m.src_hs, dst,
                                     a.out_head_stride, a.num_heads, a.rope.head_size, lane);
          break;
        case kDirectRotate:
          warp_relocate_row<T, NEOX ? 1 : 2, NEOX, false>(
              reinterpret_cast<const T*>(m.src), m.src_hs / (int64_t)sizeof(T),
              reinterpret_cast<T*>(dst), dst_hs, a.num_heads, a.rope.head_size,
              a.rope.rotary_dim, rope_row<T>(a.rope, m.old_pos), rope_row<T>(a.rope, t), lane);
          break;
        default:
          warp_zero_heads<16>(dst, a.out_head_stride, a.num_heads, units, lane);
          break;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
}


// ---- bulk-store variant (staging rows contiguous) ---------------------------
// Same tiles, classification and ring as blend_load_tma_kernel, but all data
// movement is TMA: the producer stages each run of rows whose sources are
// contiguous (a reused chunk, or consecutive slots of one vLLM block) with one
// bulk load, plus one bulk load for the run's old and one for its new cos|sin
// rows; consumers only zero gap rows and relocate K in place in shared memory,
// with (row, head, pair group) items spread over all consumer threads; the
// producer then writes the finished tile with one bulk store.  A stage is
// reloaded once its store has finished reading it.
//
// Stage layout: data [rows][row_bytes] | old cos|sin [rows][cs_row] |
// new cos|sin [rows][cs_row].
template <typename T, bool NEOX>
__device__ __forceinline__ bool bulk_store_tile(const LoadArgs& a, int64_t tile, int rows_per_tile,
                                                int row_bytes, const unsigned char* stage,
                                                uint64_t* consumed, uint32_t use, int lane,
                                                int32_t* error) {
  if (!mbar_wait(consumed, use & 1u)) {
    if (lane == 0) report(error, 3);
    return false;
  }
  if (lane == 0) {
    const int plane = static_cast<int>(tile & 1);
    const int64_t tok0 = (tile >> 1) * rows_per_tile;
    const int64_t rows = min(static_cast<int64_t>(rows_per_tile), a.alloc_end - tok0);
    bulk_store(a.out + plane * a.out_plane_stride + tok0 * row_bytes, stage,
               static_cast<uint32_t>(rows * row_bytes));
    bulk_commit();
  }
  __syncwarp();
  return true;
}

// Shared memory of one CTA: S stages of tile_bytes, row metadata, barriers,
// and the segment table when it is small enough.
inline size_t bulk_smem_bytes(int stages, int tile_bytes, int64_t num_segments) {
  return static_cast<size_t>(stages) * tile_bytes + stages * kMaxRows * sizeof(RowMeta) +
         2 * stages * sizeof(uint64_t) +
         (num_segments <= kSmemSegments ? num_segments * sizeof(cb_segment_t) : 0);
}

// S stages; tile j - LAG is stored after tile j's loads are issued, so LAG
// tiles of loads stay in flight while the consumers work.
template <typename T, bool NEOX, int S, int LAG>
__global__ void __launch_bounds__(kThreads, 3) blend_load_bulk_kernel(LoadArgs a, int rows_per_tile,
                                                                    int tile_bytes, int64_t tiles,
                                                                    int32_t* error) {
  static_assert(LAG >= 1 && LAG <= S - 1, "store lag must leave a stage to load into");
  constexpr int kStages = S;
  constexpr int kStoreLag = LAG;
  const int kTileBytes = tile_bytes;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ring = smem;
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + kStages * kTileBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + kStages * kMaxRows);
  uint64_t* consumed = full + kStages;
  cb_segment_t* seg_smem = reinterpret_cast<cb_segment_t*>(consumed + kStages);
  constexpr int E = 16 / sizeof(T);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head_bytes = a.rope.head_size * static_cast<int>(sizeof(T));
  const int row_bytes = a.num_heads * head_bytes;
  const int cs_row = a.rope.rotary_dim * static_cast<int>(sizeof(T));
  const int old_off = rows_per_tile * row_bytes;
  const int new_off = old_off + rows_per_tile * cs_row;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&consumed[st], kConsumerWarps);
    }
    mbar_init_fence();
  }
  const bool segs_in_smem = a.num_segments <= kSmemSegments;
  if (segs_in_smem) {
    const int words = static_cast<int>(a.num_segments * sizeof(cb_segment_t) / sizeof(uint2));
    const uint2* from = reinterpret_cast<const uint2*>(a.segments);
    uint2* to = reinterpret_cast<uint2*>(seg_smem);
    for (int i = threadIdx.x; i < words; i += blockDim.x) to[i] = from[i];
  }
  __syncthreads();
  const cb_segment_t* segs = segs_in_smem ? seg_smem : a.segments;

  if (warp == 0) {
    // ---- producer: classify, stage runs with bulk loads, store finished tiles
    RowRaw raw[2], raw_next[2];
    {
      const int64_t tok0 = (static_cast<int64_t>(blockIdx.x) >> 1) * rows_per_tile;
      raw[0] = load_raw(a, blockIdx.x < tiles && lane < rows_per_tile ? tok0 + lane : a.alloc_end);
      raw[1] = load_raw(a, blockIdx.x < tiles && lane + 32 < rows_per_tile ? tok0 + lane + 32
                                                                             : a.alloc_end);
    }
    bool ok = true;
    uint32_t j = 0;
    for (int64_t tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++j) {
      const int st = static_cast<int>(j % kStages);
      const int64_t next = tile + gridDim.x;
      const int64_t next0 = (next >> 1) * rows_per_tile;
      raw_next[0] = load_raw(a, next < tiles && lane < rows_per_tile ? next0 + lane : a.alloc_end);
      raw_next[1] = load_raw(a, next < tiles && lane + 32 < rows_per_tile ? next0 + lane + 32
                                                                           : a.alloc_end);
      // the store that last read this stage (tile j - kStages) must be done
      // reading; only the kStages - kStoreLag - 1 stores issued after it may not be
      if (lane == 0 && j >= static_cast<uint32_t>(kStages))
        bulk_wait_read<kStages - kStoreLag - 1>();
      __syncwarp();
      const int plane = static_cast<int>(tile & 1);
      const int64_t tok0 = (tile >> 1) * rows_per_tile;
      const int nrows = static_cast<int>(min(static_cast<int64_t>(rows_per_tile), a.alloc_end - tok0));
      unsigned char* stage = ring + st * kTileBytes;
      RowMeta mq[2];
      uint32_t bytes = 0;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int r = lane + 32 * q;
        mq[q] = RowMeta{0, 0, kNone, 0};
        if (r < nrows) {
          mq[q] = classify_row(a, segs, plane, tok0 + r, raw[q], head_bytes, sizeof(T));
          meta[st * kMaxRows + r] = mq[q];
          if (mq[q].kind == kSmemCopy) bytes += row_bytes;
          if (mq[q].kind == kSmemRotate) bytes += row_bytes + 2 * cs_row;
        }
      }
      raw[0] = raw_next[0];
      raw[1] = raw_next[1];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
      __syncwarp();
      if (lane == 0) {
        if (bytes)
          mbar_arrive_expect_tx(&full[st], bytes);
        else
          mbar_arrive(&full[st]);
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (32 * q >= nrows) break;
        const RowMeta m = mq[q];
        const bool staged = m.kind == kSmemCopy || m.kind == kSmemRotate;
        const bool whole = m.src_hs == head_bytes;  // heads back to back: one copy per row
        const int64_t prev_src = __shfl_up_sync(0xffffffffu, m.src, 1);
        const int prev_kind = __shfl_up_sync(0xffffffffu, m.kind, 1);
        const int prev_pos = __shfl_up_sync(0xffffffffu, m.old_pos, 1);
        const int prev_whole = __shfl_up_sync(0xffffffffu, whole ? 1 : 0, 1);
        const bool joins = lane > 0 && staged && whole && prev_whole && prev_kind == m.kind &&
                           m.src == prev_src + row_bytes &&
                           (m.kind != kSmemRotate || m.old_pos == prev_pos + 1);
        const bool head = staged && !joins;
        const uint32_t heads = __ballot_sync(0xffffffffu, head);
        const uint32_t staged_mask = __ballot_sync(0xffffffffu, staged);
        if (!head) continue;
        const uint32_t above = lane == 31 ? 0u : (0xffffffffu << (lane + 1));
        const uint32_t stops = (heads | ~staged_mask) & above;
        const int end = stops ? __ffs(stops) - 1 : 32;
        const int len = end - lane;
        const int r = lane + 32 * q;
        unsigned char* dst = stage + r * row_bytes;
        if (whole) {
          bulk_load(dst, reinterpret_cast<const void*>(m.src), len * row_bytes, &full[st]);
        } else {
          for (int h = 0; h < a.num_heads; ++h)  // len == 1: head-strided rows never join
            bulk_load(dst + h * head_bytes, reinterpret_cast<const void*>(m.src + h * m.src_hs),
                      head_bytes, &full[st]);
        }
        if (m.kind == kSmemRotate) {
          bulk_load(stage + old_off + r * cs_row, rope_row<T>(a.rope, m.old_pos), len * cs_row,
                    &full[st]);
          bulk_load(stage + new_off + r * cs_row, rope_row<T>(a.rope, tok0 + r), len * cs_row,
                    &full[st]);
        }
      }
      if (j >= static_cast<uint32_t>(kStoreLag)) {
        const uint32_t u = j - kStoreLag;
        ok = bulk_store_tile<T, NEOX>(a, blockIdx.x + static_cast<int64_t>(u) * gridDim.x,
                                      rows_per_tile, row_bytes,
                                      ring + (u % kStages) * kTileBytes, &consumed[u % kStages],
                                      u / kStages, lane, error);
      }
    }
    const uint32_t first = j > static_cast<uint32_t>(kStoreLag) ? j - kStoreLag : 0u;
    for (uint32_t u = first; u < j; ++u) {
      if (ok) {
        ok = bulk_store_tile<T, NEOX>(a, blockIdx.x + static_cast<int64_t>(u) * gridDim.x,
                                      rows_per_tile, row_bytes,
                                      ring + (u % kStages) * kTileBytes, &consumed[u % kStages],
                                      u / kStages, lane, error);
      } else {
        // after a failed wait: give the loads still in flight (bounded) time to land
        mbar_wait(&full[u % kStages], (u / kStages) & 1u);
      }
    }
    if (lane == 0) bulk_wait<0>();
    return;
  }

  // ---- consumers: zero gaps, unaligned rows, in-place relocation
  const int cw = warp - 1;
  const int ct = threadIdx.x - 32;
  constexpr int kConsumerThreads = 32 * kConsumerWarps;
  const int rot_items = NEOX ? a.rope.rotary_dim / 2 / E : a.rope.rotary_dim / E;
  const int items_per_row = a.num_heads * rot_items;
  const int units = head_bytes / 16;
  uint32_t j = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
    const int st = static_cast<int>(j % kStages);
    if (!mbar_wait(&full[st], (j / kStages) & 1u)) {
      if (lane == 0) report(error, 2);
      return;
    }
    const int plane = static_cast<int>(tile & 1);
    const int64_t tok0 = (tile >> 1) * rows_per_tile;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(rows_per_tile), a.alloc_end - tok0));
    unsigned char* stage = ring + st * kTileBytes;
    const RowMeta* tm = meta + st * kMaxRows;
    for (int r = cw; r < nrows; r += kConsumerWarps) {
      const RowMeta m = tm[r];
      char* row = reinterpret_cast<char*>(stage + r * row_bytes);
      switch (m.kind) {
        case kSmemCopy:
        case kSmemRotate:
          break;
        case kDirectCopy:
          warp_copy_heads<sizeof(T)>(reinterpret_cast<const char*>(m.src), m.src_hs, row,
                                     head_bytes, a.num_heads, a.rope.head_size, lane);
          break;
        case kDirectRotate:
          warp_relocate_row<T, NEOX ? 1 : 2, NEOX, false>(
              reinterpret_cast<const T*>(m.src), m.src_hs / (int64_t)sizeof(T),
              reinterpret_cast<T*>(row), a.rope.head_size, a.num_heads, a.rope.head_size,
              a.rope.rotary_dim, rope_row<T>(a.rope, m.old_pos), rope_row<T>(a.rope, tok0 + r),
              lane);
          break;
        default:
          warp_zero_heads<16>(row, head_bytes, a.num_heads, units, lane);
          break;
      }
    }
    if (plane == 0) {
      const int total = nrows * items_per_row;
      for (int i = ct; i < total; i += kConsumerThreads) {
        const int r = i / items_per_row;
        if (tm[r].kind != kSmemRotate) continue;
        const int c = i - r * items_per_row;
        const int h = c / rot_items;
        const int k = c - h * rot_items;
        T* x = reinterpret_cast<T*>(stage + r * row_bytes + h * head_bytes);
        relocate_item<T, E, NEOX, true>(x, x, k, a.rope.rotary_dim,
                                        reinterpret_cast<const T*>(stage + old_off + r * cs_row),
                                        reinterpret_cast<const T*>(stage + new_off + r * cs_row));
      }
    }
    fence_async_smem();  // generic-proxy writes above -> the producer's bulk store
    __syncwarp();
    if (lane == 0) mbar_arrive(&consumed[st]);
  }
}


// ---- flat variant (rows under 1 KiB: one or a few heads per rank) ----------
// One thread per 16-byte work item of one row: a rotary item (NEOX: E
// consecutive pairs, i.e. one vector in each half; GPT-J: one vector of E/2
// pairs) or a pass-through / V-plane vector.  No tiles, no barriers: with rows
// this small a tile pipeline does a few latency-bound round trips per CTA,
// while here every thread has its loads in flight at once.  Rows are
// classified exactly as by the tile kernels (classify_row).
template <typename T, bool NEOX>
__global__ void __launch_bounds__(256) blend_load_flat_kernel(LoadArgs a) {
  constexpr int E = 16 / sizeof(T);
  const int D = a.rope.head_size;
  const int R = a.rope.rotary_dim;
  const int half = R / 2;
  const int rot_items = NEOX ? R / 2 / E : R / E;
  const uint32_t k_items = static_cast<uint32_t>(rot_items + (D - R) / E);  // per head, K plane
  const uint32_t v_items = static_cast<uint32_t>(D / E);                    // per head, V plane
  const uint32_t k_row = a.num_heads * k_items;
  const uint32_t v_row = a.num_heads * v_items;
  const uint32_t nk = static_cast<uint32_t>(a.alloc_end) * k_row;
  const uint32_t total = nk + static_cast<uint32_t>(a.alloc_end) * v_row;
  const int head_bytes = D * static_cast<int>(sizeof(T));
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    int plane;
    uint32_t t, h, c;
    if (i < nk) {
      plane = 0;
      t = i / k_row;
      const uint32_t r = i - t * k_row;
      h = r / k_items;
      c = r - h * k_items;
    } else {
      plane = 1;
      const uint32_t j = i - nk;
      t = j / v_row;
      const uint32_t r = j - t * v_row;
      h = r / v_items;
      c = r - h * v_items;
    }
    const RowMeta m = classify_row(a, a.segments, plane, t, load_raw(a, t), head_bytes, sizeof(T));
    T* d = reinterpret_cast<T*>(a.out + plane * a.out_plane_stride + t * a.out_token_stride +
                                h * a.out_head_stride);
    // element offsets of this item: one vector, or (NEOX rotary) one in each half
    const bool pair = plane == 0 && NEOX && static_cast<int>(c) < rot_items;
    const int off0 = plane == 1 ? static_cast<int>(c) * E
                     : static_cast<int>(c) < rot_items ? static_cast<int>(c) * E
                                                       : R + (static_cast<int>(c) - rot_items) * E;
    if (m.kind == kZero) {
      Pack<T, E> z;
#pragma unroll
      for (int e = 0; e < E; ++e) z.v[e] = Elem<T>::from_f(0.0f);
      store_pack<T, E, true>(d + off0, z);
      if (pair) store_pack<T, E, true>(d + half + off0, z);
      continue;
    }
    const T* s = reinterpret_cast<const T*>(m.src + static_cast<int64_t>(h) * m.src_hs);
    const bool aligned = m.kind == kSmemCopy || m.kind == kSmemRotate;
    const bool rotate = (m.kind == kSmemRotate || m.kind == kDirectRotate) &&
                        static_cast<int>(c) < rot_items;
    if (rotate) {
      const T* old_cs = rope_row<T>(a.rope, m.old_pos);
      const T* new_cs = rope_row<T>(a.rope, t);
      if (aligned)
        relocate_item<T, E, NEOX, true>(s, d, static_cast<int>(c), R, old_cs, new_cs);
      else
        relocate_item<T, E, NEOX, false>(s, d, static_cast<int>(c), R, old_cs, new_cs);
      continue;
    }
    if (aligned) {
      store_pack<T, E, true>(d + off0, load_pack<T, E, true>(s + off0));
      if (pair) store_pack<T, E, true>(d + half + off0, load_pack<T, E, true>(s + half + off0));
    } else {
      store_pack<T, E, true>(d + off0, load_pack<T, E, false>(s + off0));
      if (pair) store_pack<T, E, true>(d + half + off0, load_pack<T, E, false>(s + half + off0));
    }
  }
}

}  // namespace tma

struct RelocArgs {
  const char* key;
  char* out;
  int64_t token_stride;
  int64_t out_token_stride;
  int64_t num_tokens;
  int num_heads;
  const int64_t* old_pos;
  const int64_t* new_pos;
  RopeDesc rope;
};

template <typename T, int E, bool NEOX>
__global__ void __launch_bounds__(256) relocate_kernel(RelocArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = warp; t < a.num_tokens; t += nwarps) {
    const int64_t op = __ldg(a.old_pos + t);
    const int64_t np = __ldg(a.new_pos + t);
    if (op < 0 || op >= a.rope.max_position || np < 0 || np >= a.rope.max_position) continue;
    warp_relocate_row<T, E, NEOX, E * sizeof(T) == 16>(
        reinterpret_cast<const T*>(a.key + t * a.token_stride), a.rope.head_size,
        reinterpret_cast<T*>(a.out + t * a.out_token_stride), a.rope.head_size, a.num_heads,
        a.rope.head_size, a.rope.rotary_dim, rope_row<T>(a.rope, op), rope_row<T>(a.rope, np),
        lane);
  }
}

inline int grid_for(int64_t warps) {
  const int64_t blocks = (warps + 7) / 8;
  return static_cast<int>(blocks < kSmCount * 8 ? blocks : kSmCount * 8);
}

// Chooses the 16-byte path when every address, stride and rotary split
// allows it; otherwise the scalar path.
bool use_vector_path(uint64_t addr_acc, int esize, int head_size, int rotary_dim, bool neox) {
  const int E = 16 / esize;
  if (vector_bytes(addr_acc) < 16) return false;
  if ((head_size * esize) % 16) return false;
  if ((rotary_dim * esize) % 16) return false;
  if (neox ? ((rotary_dim / 2) % E) : (rotary_dim % E)) return false;
  if ((head_size - rotary_dim) % E) return false;
  return true;
}

// Bulk-store load: tile size, ring depth, store lag and CTAs per SM.
// CB_LOAD_VARIANT selects a fixed configuration (tuning sweeps only).
#ifndef CB_LOAD_VARIANT
#define CB_LOAD_VARIANT 0
#endif
// CB_LOAD_CTAS > 0 overrides the bulk kernel's CTAs per SM, CB_FLAT_BLOCKS > 0
// the flat kernel's 256-thread blocks per SM, CB_TMA_LOAD_CTAS > 0 the tile
// kernel's CTAs per SM (tuning sweeps only).
#ifndef CB_LOAD_CTAS
#define CB_LOAD_CTAS 0
#endif
#ifndef CB_FLAT_BLOCKS
#define CB_FLAT_BLOCKS 0
#endif
#ifndef CB_TMA_LOAD_CTAS
#define CB_TMA_LOAD_CTAS 0
#endif
// CB_FLAT_BELOW: row bytes under which the flat kernel loads (tuning sweeps only)
#ifndef CB_FLAT_BELOW
#define CB_FLAT_BELOW 1024
#endif

template <typename T, bool NEOX, int S, int LAG>
int launch_bulk_variant(const LoadArgs& a, int tile_bytes, int ctas_per_sm, int row_bytes,
                        int cs_bytes, int32_t* error, cudaStream_t s) {
  int rows = tile_bytes / (row_bytes + cs_bytes);
  if (rows > tma::kMaxRows) rows = tma::kMaxRows;
  const int64_t tiles = 2 * ((a.alloc_end + rows - 1) / rows);
  if (CB_LOAD_CTAS > 0) ctas_per_sm = CB_LOAD_CTAS;
  const int64_t cap = static_cast<int64_t>(kSmCount) * ctas_per_sm;
  const int grid = static_cast<int>(tiles < cap ? tiles : cap);
  auto kernel = tma::blend_load_bulk_kernel<T, NEOX, S, LAG>;
  const size_t smem = tma::bulk_smem_bytes(S, tile_bytes, a.num_segments);
  const int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
  if (rc != CB_OK) return rc;
  kernel<<<grid, tma::kThreads, smem, s>>>(a, rows, tile_bytes, tiles, error);
  return launch_status("cb_blend_load_layer");
}

template <typename T, bool NEOX>
int launch_bulk_load(const LoadArgs& a, int row_bytes, int cs_bytes, int32_t* error,
                     cudaStream_t s) {
  switch (CB_LOAD_VARIANT) {
    case 1: return launch_bulk_variant<T, NEOX, 3, 1>(a, 20480, 3, row_bytes, cs_bytes, error, s);
    case 2: return launch_bulk_variant<T, NEOX, 4, 2>(a, 20480, 2, row_bytes, cs_bytes, error, s);
    case 3: return launch_bulk_variant<T, NEOX, 4, 2>(a, 16384, 3, row_bytes, cs_bytes, error, s);
    case 5: return launch_bulk_variant<T, NEOX, 3, 2>(a, 32768, 2, row_bytes, cs_bytes, error, s);
    default: break;
  }
  // measured on B200 (config-2 request, per-rank shards of TP2..TP8)
  if (row_bytes >= 1024)
    return launch_bulk_variant<T, NEOX, 3, 2>(a, 32768, 2, row_bytes, cs_bytes, error, s);
  return launch_bulk_variant<T, NEOX, 3, 1>(a, 20480, 3, row_bytes, cs_bytes, error, s);
}

template <typename T, bool NEOX>
int launch_tma_load(const LoadArgs& a, int32_t* error, cudaStream_t s) {
  const int row_bytes = a.num_heads * a.rope.head_size * static_cast<int>(sizeof(T));
  const int cs_bytes = 2 * a.rope.rotary_dim * static_cast<int>(sizeof(T));
  int rows = tma::kTileBytes / (row_bytes + cs_bytes);
  if (rows > tma::kMaxRows) rows = tma::kMaxRows;
  const int64_t tiles = 2 * ((a.alloc_end + rows - 1) / rows);
  const int64_t cap = static_cast<int64_t>(kSmCount) * (CB_TMA_LOAD_CTAS > 0 ? CB_TMA_LOAD_CTAS : 3);
  const int grid = static_cast<int>(tiles < cap ? tiles : cap);
  // Staging rows back to back (the loader's [2, alloc_end, H, D] staging) and
  // rows below 2 KiB: every tile leaves shared memory as one bulk store.  For
  // wider rows the consumers' direct stores keep more loads in flight per
  // stage and measured faster (B200, 8 heads x 128: 41.8 vs 44.5 us).
  const bool dense_out = a.out_token_stride == row_bytes &&
                         a.out_head_stride == a.rope.head_size * static_cast<int64_t>(sizeof(T));
  if (dense_out && (row_bytes < 2048 || CB_LOAD_VARIANT != 0))
    return launch_bulk_load<T, NEOX>(a, row_bytes, cs_bytes, error, s);
  auto kernel = tma::blend_load_tma_kernel<T, NEOX>;
  const size_t smem = tma::smem_bytes(a.num_segments);
  const int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
  if (rc != CB_OK) return rc;
  kernel<<<grid, tma::kThreads, smem, s>>>(a, rows, tiles, error);
  return launch_status("cb_blend_load_layer");
}

template <typename T>
int dispatch_load(const LoadArgs& a, bool vec, bool neox, int64_t max_ctas, int32_t* error,
                  cudaStream_t s) {
  const int64_t row_bytes = (int64_t)a.num_heads * a.rope.head_size * (int64_t)sizeof(T);
  const int64_t cs_bytes = 2 * (int64_t)a.rope.rotary_dim * (int64_t)sizeof(T);
  const int64_t flat_items = a.alloc_end * (2 * row_bytes / 16);
  const bool flat_ok = flat_items < (int64_t(1) << 31);
  if (vec && max_ctas <= 0 && flat_ok && (row_bytes < CB_FLAT_BELOW || CB_LOAD_VARIANT == 9)) {
    // device-memory sources, rows under 1 KiB: one thread per 16-byte item
    const int64_t blocks = (flat_items + 255) / 256;
    const int64_t cap = (int64_t)kSmCount * (CB_FLAT_BLOCKS > 0 ? CB_FLAT_BLOCKS : 8);
    const int grid = static_cast<int>(blocks < cap ? blocks : cap);
    if (neox)
      tma::blend_load_flat_kernel<T, true><<<grid, 256, 0, s>>>(a);
    else
      tma::blend_load_flat_kernel<T, false><<<grid, 256, 0, s>>>(a);
    return launch_status("cb_blend_load_layer");
  }
  if (vec && max_ctas <= 0 && row_bytes + cs_bytes <= tma::kTileBytes) {
    // device-memory sources: TMA-staged pipeline
    return neox ? launch_tma_load<T, true>(a, error, s) : launch_tma_load<T, false>(a, error, s);
  }
  int grid = grid_for(2 * a.alloc_end);
  if (max_ctas > 0 && grid > max_ctas) grid = static_cast<int>(max_ctas);
  constexpr int EV = 16 / sizeof(T);
  if (vec) {
    if (neox)
      blend_load_kernel<T, EV, true><<<grid, 256, 0, s>>>(a);
    else
      blend_load_kernel<T, EV, false><<<grid, 256, 0, s>>>(a);
  } else {
    if (neox)
      blend_load_kernel<T, 1, true><<<grid, 256, 0, s>>>(a);
    else
      blend_load_kernel<T, 2, false><<<grid, 256, 0, s>>>(a);
  }
  return launch_status("cb_blend_load_layer");
}

template <typename T>
int dispatch_reloc(const RelocArgs& a, bool vec, bool neox, cudaStream_t s) {
  const int grid = grid_for(a.num_tokens);
  constexpr int EV = 16 / sizeof(T);
  if (vec) {
    if (neox)
      relocate_kernel<T, EV, true><<<grid, 256, 0, s>>>(a);
    else
      relocate_kernel<T, EV, false><<<grid, 256, 0, s>>>(a);
  } else {
    if (neox)
      relocate_kernel<T, 1, true><<<grid, 256, 0, s>>>(a);
    else
      relocate_kernel<T, 2, false><<<grid, 256, 0, s>>>(a);
  }
  return launch_status("cb_relocate_key");
}

int check_rope(int64_t head_size, int64_t rotary_dim, int is_neox, int dtype) {
  CB_REQUIRE(dtype_bytes(dtype) > 0, "unsupported dtype %d", dtype);
  CB_REQUIRE(head_size > 0 && head_size < 65536, "head_size out of range");
  CB_REQUIRE(rotary_dim > 0 && rotary_dim <= head_size && rotary_dim % 2 == 0,
             "rotary_dim must be even and within head_size");
  // The GPT-J scalar path moves (even, odd) element pairs.
  CB_REQUIRE(is_neox || head_size % 2 == 0, "GPT-J style RoPE needs an even head_size");
  return CB_OK;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_relocate_key(const void* key, void* out, int64_t token_stride,
                               int64_t out_token_stride, int64_t num_tokens, int64_t num_heads,
                               int64_t head_size, int64_t rotary_dim, int is_neox, int dtype,
                               const void* cos_sin, int64_t max_position,
                               const int64_t* old_positions, const int64_t* new_positions,
                               void* stream) {
  CB_BIND(stream, out);
  int rc = check_rope(head_size, rotary_dim, is_neox, dtype);
  if (rc != CB_OK) return rc;
  CB_REQUIRE(num_tokens >= 0 && num_heads > 0, "bad token/head count");
  if (num_tokens == 0) return CB_OK;
  CB_REQUIRE(key && out && cos_sin && old_positions && new_positions, "null pointer argument");
  CB_REQUIRE(max_position > 0, "empty cos_sin cache");
  const int esize = dtype_bytes(dtype);
  RelocArgs a{static_cast<const char*>(key),
              static_cast<char*>(out),
              token_stride,
              out_token_stride,
              num_tokens,
              static_cast<int>(num_heads),
              old_positions,
              new_positions,
              {cos_sin, max_position, static_cast<int>(rotary_dim), static_cast<int>(head_size)}};
  const uint64_t acc = reinterpret_cast<uint64_t>(key) | reinterpret_cast<uint64_t>(out) |
                       (uint64_t)token_stride | (uint64_t)out_token_stride |
                       reinterpret_cast<uint64_t>(cos_sin);
  const bool vec = use_vector_path(acc, esize, (int)head_size, (int)rotary_dim, is_neox != 0);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CB_DTYPE_BF16:
      return dispatch_reloc<__nv_bfloat16>(a, vec, is_neox != 0, s);
    case CB_DTYPE_FP16:
      return dispatch_reloc<__half>(a, vec, is_neox != 0, s);
    default:
      return dispatch_reloc<float>(a, vec, is_neox != 0, s);
  }
}

extern "C" int cb_blend_load_layer(void* out, int64_t out_plane_stride, int64_t out_token_stride,
                                   int64_t out_head_stride, int64_t alloc_end, int64_t apc_prefix,
                                   const void* k_cache, const void* v_cache, int64_t block_stride,
                                   int64_t slot_stride, int64_t head_stride, int64_t num_blocks,
                                   int64_t block_size, const int64_t* slots, int64_t num_heads,
                                   int64_t head_size, int dtype, const int32_t* token_segment,
                                   const cb_segment_t* segments, int64_t num_segments,
                                   const void* cos_sin, int64_t max_position, int64_t rotary_dim,
                                   int is_neox, int64_t max_ctas, int32_t* device_error,
                                   void* stream) {
  CB_BIND(stream, out);
  int rc = check_rope(head_size, rotary_dim, is_neox, dtype);
  if (rc != CB_OK) return rc;
  CB_REQUIRE(alloc_end >= 0 && alloc_end < (int64_t(1) << 30), "alloc_end out of range");
  CB_REQUIRE(apc_prefix >= 0 && apc_prefix <= alloc_end, "apc_prefix out of range");
  CB_REQUIRE(num_heads > 0 && num_heads * head_size < (int64_t(1) << 24), "bad head count");
  if (alloc_end == 0) return CB_OK;
  CB_REQUIRE(out != nullptr, "null output");
  if (apc_prefix > 0) {
    CB_REQUIRE(k_cache && v_cache && slots, "APC prefix needs the paged cache and slots");
    CB_REQUIRE(num_blocks > 0 && block_size > 0 && num_blocks * block_size < (int64_t(1) << 31),
               "bad paged pool");
  }
  if (apc_prefix < alloc_end) CB_REQUIRE(token_segment != nullptr, "null token_segment");
  CB_REQUIRE(num_segments == 0 || segments != nullptr, "null segments");
  CB_REQUIRE(num_segments == 0 || cos_sin != nullptr, "segments need a cos_sin cache");
  const int esize = dtype_bytes(dtype);
  LoadArgs a{static_cast<char*>(out),
             out_plane_stride,
             out_token_stride,
             out_head_stride,
             alloc_end,
             apc_prefix,
             static_cast<const char*>(k_cache),
             static_cast<const char*>(v_cache),
             block_stride,
             slot_stride,
             head_stride,
             num_blocks * block_size,
             static_cast<uint32_t>(block_size > 0 ? block_size : 1),
             slots,
             static_cast<int>(num_heads),
             token_segment,
             segments,
             num_segments,
             {cos_sin, max_position, static_cast<int>(rotary_dim), static_cast<int>(head_size)}};
  // Segment source addresses are validated for alignment by the host
  // wrapper (it only builds 16-byte aligned descriptors on the vector path);
  // here the staging and paged strides decide.
  uint64_t acc = reinterpret_cast<uint64_t>(out) | (uint64_t)out_plane_stride |
                 (uint64_t)out_token_stride | (uint64_t)out_head_stride |
                 reinterpret_cast<uint64_t>(cos_sin);
  if (apc_prefix > 0)
    acc |= reinterpret_cast<uint64_t>(k_cache) | reinterpret_cast<uint64_t>(v_cache) |
           (uint64_t)block_stride | (uint64_t)slot_stride | (uint64_t)head_stride;
  const bool vec = use_vector_path(acc, esize, (int)head_size, (int)rotary_dim, is_neox != 0);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CB_DTYPE_BF16:
      return dispatch_load<__nv_bfloat16>(a, vec, is_neox != 0, max_ctas, device_error, s);
    case CB_DTYPE_FP16:
      return dispatch_load<__half>(a, vec, is_neox != 0, max_ctas, device_error, s);
    default:
      return dispatch_load<float>(a, vec, is_neox != 0, max_ctas, device_error, s);
  }
}
