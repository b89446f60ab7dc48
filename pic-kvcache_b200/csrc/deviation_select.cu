// K3: K-deviation scoring and masked radix top-k selection.
//
// kv_deviation (cacheblend_vllm/ascend.py:535-538):
//   score[i] = sum_j (float(k_fresh[i, j]) - float(k_cached[abs_i, j]))^2
// HBM-bound: 2 x width x esize bytes read and 4 bytes written per token.  One
// warp per token; the reduction order is fixed so that the CPU oracle
// reproduces the scores bit for bit: lane l owns units (16-byte vectors, or
// single elements on the unaligned path) l, l+32, l+64, ... and accumulates
// d = fresh - cached (fp32, RN) as acc = fmaf(d, d, acc) element by element;
// then acc += shfl_xor(acc, o) for o = 16, 8, 4, 2, 1.
//
// select_topk (_select, cacheblend_vllm/ascend.py:757-796 after the
// all-reduce): ascending indices of base ∪ top-k(non-base scores).  One CTA
// of 1024 threads: four 8-bit radix passes over order-preserving keys find the
// k-th largest key T and how many entries equal to T to keep (lowest indices
// first); a two-pass ordered compaction writes the indices.  Scores are small
// (<= 4 B x active tokens) and L2-resident, so the select is latency-bound.
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <tuple>

#include <string.h>

#include "cb_async.cuh"
#include "cb_common.cuh"

namespace cb {
namespace {

template <typename T, int UE>
struct Unit;  // UE elements per unit
template <typename T>
struct Unit<T, 1> {
  static __device__ __forceinline__ void acc(const char* f, const char* c, float& s) {
    const float d = __fsub_rn(Elem<T>::to_f(*reinterpret_cast<const T*>(f)),
                              Elem<T>::to_f(*reinterpret_cast<const T*>(c)));
    s = __fmaf_rn(d, d, s);
  }
};

template <typename T>
__device__ __forceinline__ void acc_vec16(const uint4& fv, const uint4& cv, float& s) {
  constexpr int N = 16 / sizeof(T);
  const T* f = reinterpret_cast<const T*>(&fv);
  const T* c = reinterpret_cast<const T*>(&cv);
#pragma unroll
  for (int e = 0; e < N; ++e) {
    const float d = __fsub_rn(Elem<T>::to_f(f[e]), Elem<T>::to_f(c[e]));
    s = __fmaf_rn(d, d, s);
  }
}

// Deviation operands of one launch.
struct DevArgs {
  const char* fresh;
  int64_t fresh_stride;
  const char* cached;
  int64_t cached_stride;
  int64_t cached_rows;
  const int64_t* abs_index;
  int64_t abs_offset;
  int64_t n;
};

// Scores every token this warp owns (tokens warp, warp + nwarps, ...): one warp
// per token, the fixed association order above; `sink(i, score)` runs on lane 0.
// A row whose cached index falls outside the cached rows scores NaN, unread.
template <typename T, bool VEC, typename Sink>
__device__ __forceinline__ void score_rows(const DevArgs& a, int width, int64_t warp, int64_t nwarps,
                                           Sink&& sink) {
  const int lane = threadIdx.x & 31;
  for (int64_t i = warp; i < a.n; i += nwarps) {
    const int64_t ai = a.abs_index ? __ldg(a.abs_index + i) : a.abs_offset + i;
    if (ai < 0 || ai >= a.cached_rows) {  // never read outside the cached rows
      if (lane == 0) sink(i, __int_as_float(0x7fc00000));
      continue;
    }
    const char* f = a.fresh + i * a.fresh_stride;
    const char* c = a.cached + ai * a.cached_stride;
    float s = 0.0f;
    if (VEC) {
      const int units = width * static_cast<int>(sizeof(T)) / 16;
      constexpr int U = 4;
      for (int u0 = lane; u0 < units; u0 += 32 * U) {
        uint4 fv[U], cv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int q = u0 + 32 * u;
          if (q < units) {
            fv[u] = ld_stream(reinterpret_cast<const uint4*>(f) + q);
            cv[u] = ld_stream(reinterpret_cast<const uint4*>(c) + q);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (u0 + 32 * u < units) acc_vec16<T>(fv[u], cv[u], s);
        }
      }
    } else {
      for (int q = lane; q < width; q += 32)
        Unit<T, 1>::acc(f + q * sizeof(T), c + q * sizeof(T), s);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) sink(i, s);
  }
}

// Rows of at most 32 16-byte units (up to two 128-dim bf16 heads per rank):
// 32 / units tokens share a warp, one unit per lane, and each lane keeps four
// tokens' loads in flight.  Same association order as score_rows: a lane's
// unit sum with fmaf, then the xor butterfly; the butterfly steps of offset >=
// units that score_rows also takes only add lanes holding +0.0 to a sum of
// squares (>= 0), so skipping them changes no bit.  `sink` runs on the lane
// holding unit 0 of each token.
template <typename T, typename Sink>
__device__ __forceinline__ void score_small_rows(const DevArgs& a, int units_log2, int64_t warp,
                                                 int64_t nwarps, Sink&& sink) {
  constexpr int R = 4;  // token groups per warp per iteration
  const int lane = threadIdx.x & 31;
  const int units = 1 << units_log2;
  const int per_warp = 32 >> units_log2;     // tokens per warp instruction
  const int sub = lane >> units_log2;        // this lane's token within the group
  const int q = lane & (units - 1);          // this lane's unit
  const int64_t step = nwarps * per_warp * R;
  for (int64_t base = warp * per_warp * R; base < a.n; base += step) {
    uint4 fv[R], cv[R];
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t i = base + r * per_warp + sub;
      ok[r] = false;
      if (i < a.n) {
        const int64_t ai = a.abs_index ? __ldg(a.abs_index + i) : a.abs_offset + i;
        ok[r] = ai >= 0 && ai < a.cached_rows;  // never read outside the cached rows
        if (ok[r]) {
          fv[r] = ld_stream(reinterpret_cast<const uint4*>(a.fresh + i * a.fresh_stride) + q);
          cv[r] = ld_stream(reinterpret_cast<const uint4*>(a.cached + ai * a.cached_stride) + q);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = 0.0f;
      if (ok[r]) acc_vec16<T>(fv[r], cv[r], v);
      for (int o = units >> 1; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
      const int64_t i = base + r * per_warp + sub;
      if (q == 0 && i < a.n) sink(i, ok[r] ? v : __int_as_float(0x7fc00000));
    }
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) deviation_kernel(DevArgs a, int width, float* __restrict__ scores) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  score_rows<T, VEC>(a, width, warp, nwarps, [&](int64_t i, float v) { scores[i] = v; });
}

template <typename T>
__global__ void __launch_bounds__(256) deviation_small_kernel(DevArgs a, int units_log2,
                                                              float* __restrict__ scores) {
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  score_small_rows<T>(a, units_log2, warp, nwarps, [&](int64_t i, float v) { scores[i] = v; });
}

// Order-preserving key: larger float -> larger key.// Order-preserving key: larger float -> larger key.  NaN (either sign) is
// the largest, -0.0 equals +0.0.
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xffffffffu;
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSelThreads = 1024;

// Block-wide exclusive scan of one int64 per thread (1024 threads).
__device__ int64_t block_exclusive_scan(int64_t v, int64_t* warp_sums, int64_t& total) {
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int64_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int64_t warp_prefix = wid ? warp_sums[wid - 1] : 0;
  total = warp_sums[31];
  __syncthreads();
  return warp_prefix + x - v;
}

__global__ void __launch_bounds__(kSelThreads) select_topk_kernel(
    const float* __restrict__ scores, const uint8_t* __restrict__ base, int64_t n, int64_t k,
    int64_t* __restrict__ out, int64_t cap) {
  __shared__ uint32_t hist[256];
  __shared__ int64_t warp_sums[32];
  __shared__ uint32_t s_digit;
  __shared__ int64_t s_above;
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  int64_t krem = k;
  if (k > 0) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      if (tid < 256) hist[tid] = 0;
      if (tid == 0) {
        // k <= #candidates makes the search below always succeed; if a caller
        // breaks that contract the threshold degrades to "keep every
        // candidate", which still writes fewer than #base + k indices.
        s_digit = 0;
        s_above = 0;
      }
      __syncthreads();
      for (int64_t i = tid; i < n; i += kSelThreads) {
        if (base[i]) continue;
        const uint32_t key = order_key(scores[i]);
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid < 32) {
        // lane L owns digits 255-8L .. 248-8L (descending)
        uint32_t local[8];
        uint32_t sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          local[j] = hist[255 - 8 * tid - j];
          sum += local[j];
        }
        // exclusive prefix over lanes = count of digits above this lane's range
        uint32_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (tid >= o) incl += y;
        }
        const uint32_t above = incl - sum;
        if ((int64_t)above < krem && (int64_t)incl >= krem) {
          uint32_t run = above;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if ((int64_t)(run + local[j]) >= krem) {
              s_digit = 255 - 8 * tid - j;
              s_above = run;
              break;
            }
            run += local[j];
          }
        }
      }
      __syncthreads();
      prefix |= s_digit << shift;
      pmask |= 255u << shift;
      krem -= s_above;
      __syncthreads();
    }
  }
  // prefix is the k-th largest key; keep every key > prefix and the first
  // krem keys == prefix in index order.  k == 0 keeps base entries only.
  const uint32_t thr = prefix;
  const int64_t k_eq = k > 0 ? krem : 0;
  const bool any = k > 0;
  const int64_t per = (n + kSelThreads - 1) / kSelThreads;
  const int64_t lo = per * tid < n ? per * tid : n;
  const int64_t hi = lo + per < n ? lo + per : n;
  int64_t c_sel = 0, c_eq = 0;
  for (int64_t i = lo; i < hi; ++i) {
    if (base[i]) {
      ++c_sel;
      continue;
    }
    if (!any) continue;
    const uint32_t key = order_key(scores[i]);
    if (key > thr)
      ++c_sel;
    else if (key == thr)
      ++c_eq;
  }
  int64_t total;
  int64_t sel_before = block_exclusive_scan(c_sel, warp_sums, total);
  int64_t eq_before = block_exclusive_scan(c_eq, warp_sums, total);
  for (int64_t i = lo; i < hi; ++i) {
    bool take;
    if (base[i]) {
      take = true;
    } else if (!any) {
      take = false;
    } else {
      const uint32_t key = order_key(scores[i]);
      if (key > thr) {
        take = true;
      } else if (key == thr) {
        take = eq_before < k_eq;
        ++eq_before;
        if (take && sel_before + eq_before - 1 < cap) out[sel_before + eq_before - 1] = i;
        continue;
      } else {
        take = false;
      }
    }
    if (take) {
      const int64_t pos = sel_before + (eq_before < k_eq ? eq_before : k_eq);
      if (pos < cap) out[pos] = i;
      ++sel_before;
    }
  }
}

// ---- cluster select ---------------------------------------------------------
// Eight CTAs of one thread-block cluster split the scores into contiguous
// slices held in shared memory as order keys (+ base flags).  Each radix pass
// builds a local 256-bin histogram, merges it into rank 0's histogram through
// distributed shared memory, and every CTA derives the same digit from it.
// The ordered compaction needs, per CTA, the selected counts of the lower
// ranks, again read through DSMEM.  Scores cross HBM/L2 once.
namespace cg = cooperative_groups;
constexpr int kClusterCtas = 8;
constexpr int kMaxSlice = 42 * 1024;  // keys per CTA: 5 bytes each in shared memory

__device__ __forceinline__ void find_digit(const uint32_t* hist, int64_t krem, uint32_t* s_digit,
                                           int64_t* s_above) {
  const int lane = threadIdx.x;  // called by warp 0
  uint32_t local[8];
  uint32_t sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    local[j] = hist[255 - 8 * lane - j];
    sum += local[j];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t above = incl - sum;
  if ((int64_t)above < krem && (int64_t)incl >= krem) {
    uint32_t run = above;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if ((int64_t)(run + local[j]) >= krem) {
        *s_digit = 255 - 8 * lane - j;
        *s_above = run;
        break;
      }
      run += local[j];
    }
  }
}

// Radix passes still to run: the digit at bits [shift, shift + width).
struct RadixPass {
  int shift;
  int width;
};
// four 8-bit digits over the whole 32-bit key
struct FullPasses {
  static constexpr int kCount = 4;
  static __device__ __forceinline__ RadixPass at(int p) { return RadixPass{24 - 8 * p, 8}; }
};
// the bits below the 11-bit first digit the fused kernel takes from its global histogram
struct TailPasses {
  static constexpr int kCount = 3;
  static __device__ __forceinline__ RadixPass at(int p) {
    return p == 0 ? RadixPass{13, 8} : (p == 1 ? RadixPass{5, 8} : RadixPass{0, 5});
  }
};

// Cluster barrier halves (PTX barrier.cluster): `arrive` at kernel start and
// `wait` just before the first access to another CTA's shared memory, which
// must not come before that CTA has started.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// The selection by one cluster of 8 CTAs (shared by select_cluster_kernel, the
// fused deviation select and the peer-exchange select): this CTA's slice of
// order keys and base flags in shared memory, the remaining radix passes, then
// the ordered compaction.  `prefix`, `pmask`, `krem`: the digits already fixed
// and the rank still sought among keys with that prefix.
//
// Every CTA pushes its local histogram of a pass into slot [its rank] of every
// CTA's inbox (DSMEM stores, 16-bit counts: a slice holds < 65,536 keys), so
// after the pass's one cluster barrier each CTA merges and searches its own
// copy from local shared memory.  The inbox is double-buffered by pass: pass
// p + 2 writes buffer p % 2 only after the barrier of pass p + 1, which every
// CTA reaches after merging pass p.  The compaction's per-CTA totals travel
// the same way, so the last barrier is the totals' one.  The caller must have
// made the cluster barrier's arrive (cluster_arrive_relaxed) once, and must not
// have waited on it: the first wait here completes it.
template <typename Passes>
__device__ __forceinline__ void cluster_select(cg::cluster_group& cluster, const float* scores,
                                               const uint8_t* base, int64_t n, int64_t k,
                                               int64_t* out, int64_t cap, int slice, uint32_t* dyn,
                                               uint32_t prefix, uint32_t pmask, int64_t krem,
                                               bool keys_ready = false) {
  const int rank = static_cast<int>(cluster.block_rank());
  uint32_t* keys = dyn;
  uint8_t* flags = reinterpret_cast<uint8_t*>(keys + slice);
  __shared__ uint32_t inbox[2][kClusterCtas][128];  // 256 16-bit counts per CTA, packed in pairs
  __shared__ uint32_t local[256];
  __shared__ uint32_t merged[256];
  __shared__ uint32_t all_totals[kClusterCtas][2];  // every CTA's (selected, tied) counts
  __shared__ int64_t warp_sums[32];
  __shared__ uint32_t s_digit;
  __shared__ int64_t s_above;
  const int tid = threadIdx.x;
  const int64_t lo = (int64_t)rank * slice;
  const int64_t hi = lo + slice < n ? lo + slice : n;
  const int m = hi > lo ? static_cast<int>(hi - lo) : 0;
  if (!keys_ready) {  // else the caller filled keys[0, m) and flags[0, m)
    for (int i = tid; i < m; i += kSelThreads) {
      keys[i] = order_key(__ldcg(scores + lo + i));  // L2: other CTAs may have just written them
      flags[i] = base[lo + i] != 0;
    }
  }
  if (tid < 256) local[tid] = 0;
  __syncthreads();
  bool waited = false;
  if (k > 0) {
#pragma unroll 1
    for (int pass = 0; pass < Passes::kCount; ++pass) {
      const RadixPass digit = Passes::at(pass);
      const int shift = digit.shift;
      const uint32_t digit_mask = (1u << digit.width) - 1u;
      if (tid == 0) {
        s_digit = 0;  // see select_topk_kernel: degrades safely if k > #candidates
        s_above = 0;
      }
      for (int i = tid; i < m; i += kSelThreads) {
        const uint32_t key = keys[i];
        if (!flags[i] && (key & pmask) == prefix) atomicAdd(&local[(key >> shift) & digit_mask], 1u);
      }
      __syncthreads();
      if (!waited) {
        cluster_wait();  // every CTA has started: its shared memory may be written
        waited = true;
      }
      if (tid < 128) {
        const uint32_t pair = local[2 * tid] | (local[2 * tid + 1] << 16);
        local[2 * tid] = 0;  // this thread's own bins: ready for the next pass
        local[2 * tid + 1] = 0;
#pragma unroll
        for (int r = 0; r < kClusterCtas; ++r) *cluster.map_shared_rank(&inbox[pass & 1][rank][tid], r) = pair;
      }
      cluster.sync();
      if (tid < 256) {
        uint32_t sum = 0;
#pragma unroll
        for (int r = 0; r < kClusterCtas; ++r) sum += (inbox[pass & 1][r][tid >> 1] >> ((tid & 1) * 16)) & 0xffffu;
        merged[tid] = sum;
      }
      __syncthreads();
      if (tid < 32) find_digit(merged, krem, &s_digit, &s_above);
      __syncthreads();
      prefix |= s_digit << shift;
      pmask |= digit_mask << shift;
      krem -= s_above;
      __syncthreads();  // all threads read s_digit before the next pass resets it
    }
  }
  if (!waited) cluster_wait();
  const uint32_t thr = prefix;
  const int64_t k_eq = k > 0 ? krem : 0;
  const bool any = k > 0;
  const int per = (m + kSelThreads - 1) / kSelThreads;
  const int a0 = per * tid < m ? per * tid : m;
  const int a1 = a0 + per < m ? a0 + per : m;
  int64_t c_sel = 0, c_eq = 0;
  for (int i = a0; i < a1; ++i) {
    if (flags[i]) {
      ++c_sel;
    } else if (any) {
      if (keys[i] > thr)
        ++c_sel;
      else if (keys[i] == thr)
        ++c_eq;
    }
  }
  // one scan of both counts: (selected << 32) | tied, neither passes 2^32 in a slice
  int64_t total;
  const int64_t before = block_exclusive_scan((c_sel << 32) | c_eq, warp_sums, total);
  if (tid < kClusterCtas) {
    uint32_t* slot = cluster.map_shared_rank(&all_totals[rank][0], tid);
    slot[0] = static_cast<uint32_t>(total >> 32);
    slot[1] = static_cast<uint32_t>(total & 0xffffffff);
  }
  cluster.sync();  // the last access to another CTA's shared memory came before this
  int64_t sel_off = 0, eq_off = 0;
  for (int r = 0; r < rank; ++r) {
    sel_off += all_totals[r][0];
    eq_off += all_totals[r][1];
  }
  int64_t sel_before = (before >> 32) + sel_off;
  int64_t eq_before = (before & 0xffffffff) + eq_off;
  for (int i = a0; i < a1; ++i) {
    const int64_t index = lo + i;
    if (flags[i] || (any && keys[i] > thr)) {
      const int64_t pos = sel_before + (eq_before < k_eq ? eq_before : k_eq);
      if (pos < cap) out[pos] = index;
      ++sel_before;
    } else if (any && keys[i] == thr) {
      if (eq_before < k_eq && sel_before + eq_before < cap) out[sel_before + eq_before] = index;
      ++eq_before;
    }
  }
}

__global__ void __launch_bounds__(kSelThreads, 1) select_cluster_kernel(
    const float* __restrict__ scores, const uint8_t* __restrict__ base, int64_t n, int64_t k,
    int64_t* __restrict__ out, int64_t cap, int slice) {
  cg::cluster_group cluster = cg::this_cluster();
  cluster_arrive_relaxed();
  extern __shared__ __align__(16) uint32_t dyn[];
  cluster_select<FullPasses>(cluster, scores, base, n, k, out, cap, slice, dyn, 0u, 0u, k);
}

// ---- fused deviation + selection ---------------------------------------------
// One launch of 8-CTA clusters for the K-deviation and the selection of a
// single-rank check layer (ascend.py:534-543 then 757-796).  Every CTA scores
// its tokens (score_rows / score_small_rows: bit-identical scores) and counts
// the non-base scores' top 11 key bits in a 2048-bin shared histogram, which it
// adds into the caller's workspace.  A cluster that has finished fences, and
// its rank 0 takes a ticket; the cluster holding the last ticket selects: the
// first digit from the global histogram, the three radix passes over the
// remaining 21 bits and the ordered compaction of cluster_select.  No CTA waits
// for another cluster, so nothing spins; the last cluster leaves the histogram
// and the ticket zeroed for the next call.
constexpr int kWideBits = 11;
constexpr int kWideBins = 1 << kWideBits;
// keys per CTA: 5 bytes each in dynamic shared memory, beside the 8 KiB histogram
constexpr int kFusedMaxSlice = 40 * 1024;

struct FusedWorkspace {
  uint32_t hist[kWideBins];
  uint32_t ticket;
};

// First (11-bit) digit from the histogram staged in shared memory: warp 0,
// lane L owns bins 2047 - 64L down to 1984 - 64L.
__device__ __forceinline__ void find_wide_digit(const uint32_t* hist, int64_t krem, uint32_t* s_digit,
                                                int64_t* s_above) {
  const int lane = threadIdx.x;
  constexpr int kPer = kWideBins / 32;
  uint32_t sum = 0;
#pragma unroll 16
  for (int j = 0; j < kPer; ++j) sum += hist[kWideBins - 1 - kPer * lane - j];
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t above = incl - sum;
  if ((int64_t)above < krem && (int64_t)incl >= krem) {
    uint32_t run = above;
    for (int j = 0; j < kPer; ++j) {
      const uint32_t count = hist[kWideBins - 1 - kPer * lane - j];
      if ((int64_t)(run + count) >= krem) {
        *s_digit = kWideBins - 1 - kPer * lane - j;
        *s_above = run;
        break;
      }
      run += count;
    }
  }
}

template <typename T, bool SMALL>
__global__ void __launch_bounds__(kSelThreads, 1) deviation_select_kernel(
    DevArgs a, int width_or_units_log2, const uint8_t* __restrict__ base, int64_t k,
    float* __restrict__ scores, int64_t* __restrict__ out, int64_t cap, int slice,
    FusedWorkspace* __restrict__ ws) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  extern __shared__ __align__(16) uint32_t dyn[];
  __shared__ uint32_t wide[kWideBins];
  __shared__ int s_last;
  __shared__ uint32_t s_digit;
  __shared__ int64_t s_above;
  const int tid = threadIdx.x;
  for (int b = tid; b < kWideBins; b += kSelThreads) wide[b] = 0;
  __syncthreads();
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + tid) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  auto sink = [&](int64_t i, float v) {
    scores[i] = v;
    if (!base[i]) atomicAdd(&wide[order_key(v) >> (32 - kWideBits)], 1u);
  };
  if (SMALL)
    score_small_rows<T>(a, width_or_units_log2, warp, nwarps, sink);
  else
    score_rows<T, true>(a, width_or_units_log2, warp, nwarps, sink);
  __syncthreads();
  for (int b = tid; b < kWideBins; b += kSelThreads)
    if (wide[b]) atomicAdd(&ws->hist[b], wide[b]);
  __threadfence();  // scores and counts visible device-wide before the ticket
  cluster.sync();
  if (rank == 0 && tid == 0) {
    const uint32_t clusters = gridDim.x / kClusterCtas;
    const int last = atomicAdd(&ws->ticket, 1u) == clusters - 1;
    for (int r = 0; r < kClusterCtas; ++r) *cluster.map_shared_rank(&s_last, r) = last;
  }
  cluster.sync();
  if (!s_last) return;
  __threadfence();
  uint32_t prefix = 0, pmask = 0;
  int64_t krem = k;
  if (k > 0) {
    // the device-wide histogram into shared memory (the CTA's own counts are flushed)
    for (int b = tid; b < kWideBins; b += kSelThreads) wide[b] = __ldcg(ws->hist + b);
    if (tid == 0) {
      s_digit = 0;
      s_above = 0;
    }
    __syncthreads();
    if (tid < 32) find_wide_digit(wide, k, &s_digit, &s_above);
    __syncthreads();
    prefix = s_digit << (32 - kWideBits);
    pmask = (uint32_t)(kWideBins - 1) << (32 - kWideBits);
    krem = k - s_above;
  }
  cluster.sync();  // every CTA of this cluster has read the histogram: clear it for the next call
  if (rank == 0) {
    for (int b = tid; b < kWideBins; b += kSelThreads) ws->hist[b] = 0;
    if (tid == 0) ws->ticket = 0;
  }
  cluster_arrive_relaxed();  // cluster_select's first wait pairs with it
  cluster_select<TailPasses>(cluster, scores, base, a.n, k, out, cap, slice, dyn, prefix, pmask, krem);
}

// ---- TP selection with the score reduction over peer memory -------------------
// `_select` after the TP all-reduce (ascend.py:764-796) with the reduction done
// in this kernel over NVLink instead of by a separate NCCL collective.  Every
// rank owns an exchange buffer that all ranks map (CUDA IPC):
//   recv  [2][world][capacity] fp32   one row per sending rank, double-buffered by call parity
//   flags [kMaxPeers][8] u32          [r][c]: calls of rank r whose slice c has landed here
//   count [8] u32                     this rank's finished calls, per cluster CTA
// Cluster CTA c owns tokens [c * slice, (c + 1) * slice): it stores its slice
// of the local partial scores into row `rank` of every rank's receive buffer
// (plain stores through the peer mapping), fences at system scope, bumps
// flag [rank][c] on every rank, waits (bounded) until every rank has bumped
// its own flags [*][c] to this call's number, then sums the rows in rank
// order -- the same fp32 order on every rank, so every rank selects the same
// tokens -- and runs the radix passes and compaction of cluster_select.
//
// A rank runs at most one call ahead of another: its call e + 1 waits for the
// other's bump of call e + 1, which the other makes only after its call e has
// read its rows.  So the rows of call e + 2 (same parity as e) never land while
// call e reads them, and two receive buffers suffice.  A wait that gives up
// records code 5 and the call goes on with whatever rows are there (its result
// is wrong, the error word says so); the flags stay consistent, because the
// late rank still makes its bump, so the next calls are right again.
//
// `emulated`: one launch plays every rank on one GPU (cluster w is rank w, all
// buffers local, partial / out / summed are [world] x their per-rank size); a
// cooperative launch, so that every cluster is resident while the others wait.
constexpr int kMaxPeers = 8;
constexpr int kPeerError = 5;

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void add_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// 64-bit scalar accesses are single-copy atomic: a word carries a score and
// the call number that wrote it, and a reader that sees the call number sees
// the score stored with it.
__device__ __forceinline__ void store_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t load_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct PeerArgs {
  uint64_t base[kMaxPeers];  // each rank's exchange buffer as mapped in this process
  int rank;
  int world;
  int emulated;
  int low_latency;           // 1: 64-bit (score, call) words, no fence or flags
  int64_t capacity;          // entries per receive row (a multiple of 4)
  int64_t flags_offset;      // bytes from a buffer's start to its flags
};

// The receive rows take 8 bytes per entry (the low-latency words; the flag
// protocol uses the first half of each parity's area as fp32 rows).
__host__ __device__ inline int64_t peer_flags_offset(int world, int64_t capacity) {
  return (int64_t)2 * world * capacity * 8;
}

__device__ __forceinline__ uint32_t* peer_flags(const PeerArgs& p, int r) {
  return reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(p.base[r]) + p.flags_offset);
}

__global__ void __launch_bounds__(kSelThreads, 1) select_peer_kernel(
    const float* __restrict__ partial, const uint8_t* __restrict__ base, int64_t n, int64_t k,
    int64_t* __restrict__ out, int64_t cap, int slice, PeerArgs peers, float* __restrict__ summed,
    int32_t* __restrict__ error) {
  cg::cluster_group cluster = cg::this_cluster();
  cluster_arrive_relaxed();  // cluster_select's first wait pairs with it
  const int crank = static_cast<int>(cluster.block_rank());
  const int me = peers.emulated ? static_cast<int>(blockIdx.x) / kClusterCtas : peers.rank;
  if (peers.emulated) {
    partial += (int64_t)me * n;
    out += (int64_t)me * cap;
    if (summed != nullptr) summed += (int64_t)me * n;
  }
  extern __shared__ __align__(16) uint32_t dyn[];
  uint32_t* keys = dyn;
  uint8_t* flags_smem = reinterpret_cast<uint8_t*>(keys + slice);
  __shared__ uint32_t s_epoch;
  const int tid = threadIdx.x;
  const int world = peers.world;
  const int64_t lo = (int64_t)crank * slice;
  const int64_t hi = lo + slice < n ? lo + slice : n;
  const int m = hi > lo ? static_cast<int>(hi - lo) : 0;
  uint32_t* my_flags = peer_flags(peers, me);
  uint32_t* my_count = my_flags + kMaxPeers * kClusterCtas;
  if (tid == 0) s_epoch = my_count[crank] + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int64_t parity = epoch & 1u;
  if (peers.low_latency) {
    // Low-latency protocol: each score crosses NVLink once, as a 64-bit word
    // (call number << 32 | score bits) in row `me` of every rank's receive
    // area; the reader polls the words themselves until they carry this call's
    // number.  No fence and no flag round trip, at twice the bytes.
    for (int i = tid; i < m; i += kSelThreads) {
      const uint64_t word = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(__ldcg(partial + lo + i));
      for (int r = 0; r < world; ++r)
        store_relaxed_sys(reinterpret_cast<uint64_t*>(peers.base[r]) + (parity * world + me) * peers.capacity + lo + i,
                          word);
    }
    const uint64_t* words = reinterpret_cast<const uint64_t*>(peers.base[me]) + parity * world * peers.capacity + lo;
    bool gave_up = false;
    const uint64_t start = async::global_ns();
    for (int i = tid; i < m; i += kSelThreads) {
      float v = 0.0f;
      for (int r = 0; r < world; ++r) {
        uint64_t w = load_relaxed_sys(words + r * peers.capacity + i);
        for (uint32_t spin = 1; static_cast<uint32_t>(w >> 32) != epoch && !gave_up; ++spin) {
          if ((spin & 63u) == 0 && async::global_ns() - start > async::kTimeoutNs) {
            gave_up = true;  // the rest of this thread's words are taken as they are
            break;
          }
          w = load_relaxed_sys(words + r * peers.capacity + i);
        }
        const float x = __uint_as_float(static_cast<uint32_t>(w));
        v = r == 0 ? x : v + x;  // rank order, as the flag protocol sums
      }
      if (summed != nullptr) summed[lo + i] = v;
      keys[i] = order_key(v);
      flags_smem[i] = base[lo + i] != 0;
    }
    if (gave_up && error != nullptr) atomicCAS(error, 0, kPeerError);
    if (tid == 0) my_count[crank] = epoch;
    cluster_select<FullPasses>(cluster, nullptr, base, n, k, out, cap, slice, dyn, 0u, 0u, k, true);
    return;
  }
  // this CTA's slice of the partial scores into row `me` of every receive buffer,
  // in 16-byte stores where both sides are aligned (slice and capacity are
  // multiples of 4 and the buffers 256-byte aligned, so that rests on `partial`)
  for (int r = 0; r < world; ++r) {
    float* row = reinterpret_cast<float*>(peers.base[r]) + (parity * world + me) * peers.capacity + lo;
    const bool vec = ((reinterpret_cast<uintptr_t>(partial + lo) | reinterpret_cast<uintptr_t>(row)) & 15) == 0;
    const int m4 = vec ? m >> 2 : 0;
    const float4* src = reinterpret_cast<const float4*>(partial + lo);
    for (int i = tid; i < m4; i += kSelThreads) reinterpret_cast<float4*>(row)[i] = src[i];
    for (int i = 4 * m4 + tid; i < m; i += kSelThreads) row[i] = partial[lo + i];
  }
  // Release: the block barrier orders every thread's stores before warp 0's
  // system-scope fence, and each flag bump follows that fence (one fence for
  // all ranks' flags; a release on every bump would wait out the NVLink round
  // trip of the bump before it).
  __syncthreads();
  if (tid < 32) {
    __threadfence_system();
    if (tid < world) add_relaxed_sys(peer_flags(peers, tid) + me * kClusterCtas + crank, 1u);
  }
  // every rank's slice `crank` of this call has landed here
  if (tid < world) {
    const uint32_t* flag = my_flags + tid * kClusterCtas + crank;
    const uint64_t start = async::global_ns();
    while (load_acquire_sys(flag) < epoch) {
      if (async::global_ns() - start > async::kTimeoutNs) {
        if (error != nullptr) atomicCAS(error, 0, kPeerError);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  const float* rows = reinterpret_cast<const float*>(peers.base[me]) + parity * world * peers.capacity + lo;
  for (int i = tid; i < m; i += kSelThreads) {
    float v = __ldcg(rows + i);
    for (int r = 1; r < world; ++r) v += __ldcg(rows + r * peers.capacity + i);
    if (summed != nullptr) summed[lo + i] = v;
    keys[i] = order_key(v);
    flags_smem[i] = base[lo + i] != 0;
  }
  if (tid == 0) my_count[crank] = epoch;
  cluster_select<FullPasses>(cluster, nullptr, base, n, k, out, cap, slice, dyn, 0u, 0u, k, true);
}

// |A n B| of two strictly ascending index lists (the two selections of the
// `compare` strategy, ascend.py:713-747): each thread binary-searches its A
// entries in B; per-warp sums, one atomic per warp.
__global__ void __launch_bounds__(256) sorted_overlap_kernel(const int64_t* __restrict__ a,
                                                             int64_t na,
                                                             const int64_t* __restrict__ b,
                                                             int64_t nb,
                                                             unsigned long long* __restrict__ count) {
  unsigned long long local = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < na; i += stride) {
    const int64_t x = __ldg(a + i);
    int64_t lo = 0, hi = nb;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (__ldg(b + mid) < x)
        lo = mid + 1;
      else
        hi = mid;
    }
    local += (lo < nb && __ldg(b + lo) == x) ? 1ull : 0ull;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(count, local);
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_kv_deviation(const void* fresh, int64_t fresh_row_stride, const void* cached,
                               int64_t cached_row_stride, int64_t cached_rows,
                               const int64_t* abs_index,
                               int64_t abs_offset, int64_t num_tokens, int64_t width, int dtype,
                               float* scores, void* stream) {
  CB_BIND(stream, scores);
  const int esize = dtype_bytes(dtype);
  CB_REQUIRE(esize > 0, "unsupported dtype %d", dtype);
  CB_REQUIRE(num_tokens >= 0 && width > 0 && width < (int64_t(1) << 24), "bad shape");
  if (num_tokens == 0) return CB_OK;
  CB_REQUIRE(fresh && cached && scores, "null pointer argument");
  CB_REQUIRE(cached_rows >= 0, "negative cached_rows");
  const uint64_t acc = reinterpret_cast<uint64_t>(fresh) | reinterpret_cast<uint64_t>(cached) |
                       (uint64_t)fresh_row_stride | (uint64_t)cached_row_stride |
                       (uint64_t)(width * esize);
  const bool vec = vector_bytes(acc) >= 16;
  const int64_t blocks = (num_tokens + 7) / 8;
  const int grid = static_cast<int>(blocks < kSmCount * 8 ? blocks : kSmCount * 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const char* f = static_cast<const char*>(fresh);
  const char* c = static_cast<const char*>(cached);
  const int w = static_cast<int>(width);
  const int64_t units = width * esize / 16;
  int units_log2 = 0;
  while ((int64_t(1) << units_log2) < units) ++units_log2;
  const bool small = vec && units <= 32 && (int64_t(1) << units_log2) == units;
  int small_grid = 0;
  if (small) {
    const int64_t per_block = 8 * (32 >> units_log2) * 4;  // tokens per block per iteration
    const int64_t small_blocks = (num_tokens + per_block - 1) / per_block;
    small_grid = static_cast<int>(small_blocks < kSmCount * 8 ? small_blocks : kSmCount * 8);
  }
#define CB_DEV_LAUNCH(T)                                                                   \
  do {                                                                                     \
    if (small)                                                                             \
      deviation_small_kernel<T><<<small_grid, 256, 0, s>>>(args, units_log2, scores);      \
    else if (vec)                                                                          \
      deviation_kernel<T, true><<<grid, 256, 0, s>>>(args, w, scores);                     \
    else                                                                                   \
      deviation_kernel<T, false><<<grid, 256, 0, s>>>(args, w, scores);                    \
  } while (0)
  const DevArgs args{f, fresh_row_stride, c, cached_row_stride, cached_rows, abs_index, abs_offset,
                     num_tokens};
  switch (dtype) {
    case CB_DTYPE_BF16:
      CB_DEV_LAUNCH(__nv_bfloat16);
      break;
    case CB_DTYPE_FP16:
      CB_DEV_LAUNCH(__half);
      break;
    default:
      CB_DEV_LAUNCH(float);
      break;
  }
#undef CB_DEV_LAUNCH
  return launch_status("cb_kv_deviation");
}

extern "C" int cb_select_topk(const float* scores, const uint8_t* base_mask, int64_t n, int64_t k,
                              int64_t* out_index, int64_t out_capacity, void* stream) {
  CB_BIND(stream, out_index);
  CB_REQUIRE(n >= 0 && k >= 0 && k <= n && out_capacity >= 0, "bad n/k");
  if (n == 0 || out_capacity == 0) return CB_OK;
  CB_REQUIRE(scores && base_mask && out_index, "null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n <= (int64_t)kClusterCtas * kMaxSlice) {
    const int slice = static_cast<int>((n + kClusterCtas - 1) / kClusterCtas);
    const size_t dyn = ((size_t)slice * 5 + 15) / 16 * 16;
    const int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(select_cluster_kernel), dyn);
    if (rc != CB_OK) return rc;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(kClusterCtas, 1, 1);
    config.blockDim = dim3(kSelThreads, 1, 1);
    config.dynamicSmemBytes = dyn;
    config.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kClusterCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.attrs = attr;
    config.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&config, select_cluster_kernel, scores, base_mask, n, k, out_index,
                           out_capacity, slice);
    if (e != cudaSuccess) {
      set_error("cb_select_topk cluster launch failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
    return launch_status("cb_select_topk");
  }
  select_topk_kernel<<<1, kSelThreads, 0, s>>>(scores, base_mask, n, k, out_index, out_capacity);
  return launch_status("cb_select_topk");
}

extern "C" int cb_sorted_overlap(const int64_t* a, int64_t na, const int64_t* b, int64_t nb,
                                 int64_t* count, void* stream) {
  CB_BIND(stream, count);
  CB_REQUIRE(na >= 0 && nb >= 0, "negative list length");
  CB_REQUIRE(count != nullptr, "null count");
  CB_REQUIRE((na == 0 || a != nullptr) && (nb == 0 || b != nullptr), "null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(count, 0, sizeof(int64_t), s);
  if (e != cudaSuccess) {
    set_error("cb_sorted_overlap: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  if (na == 0 || nb == 0) return CB_OK;
  const int64_t blocks = (na + 255) / 256;
  const int grid = static_cast<int>(blocks < kSmCount * 4 ? blocks : kSmCount * 4);
  sorted_overlap_kernel<<<grid, 256, 0, s>>>(a, na, b, nb,
                                             reinterpret_cast<unsigned long long*>(count));
  return launch_status("cb_sorted_overlap");
}

namespace {
// Clusters of deviation_select_kernel the current device runs at once (queried
// once per context, kernel and shared-memory size; 16 if the query fails).
int resident_clusters(bool small, int dtype, size_t dyn) {
  static std::mutex lock;
  static std::map<std::tuple<void*, const void*, size_t>, int> known;
  const void* fn = nullptr;
  switch (dtype) {
    case CB_DTYPE_BF16:
      fn = small ? (const void*)deviation_select_kernel<__nv_bfloat16, true>
                 : (const void*)deviation_select_kernel<__nv_bfloat16, false>;
      break;
    case CB_DTYPE_FP16:
      fn = small ? (const void*)deviation_select_kernel<__half, true>
                 : (const void*)deviation_select_kernel<__half, false>;
      break;
    default:
      fn = small ? (const void*)deviation_select_kernel<float, true>
                 : (const void*)deviation_select_kernel<float, false>;
      break;
  }
  void* context = nullptr;
  if (current_context(&context) != CB_OK) return 16;
  std::lock_guard<std::mutex> guard(lock);
  const auto key = std::make_tuple(context, fn, dyn);
  const auto it = known.find(key);
  if (it != known.end()) return it->second;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(kClusterCtas, 1, 1);
  config.blockDim = dim3(kSelThreads, 1, 1);
  config.dynamicSmemBytes = dyn;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  int count = 0;
  if (cudaOccupancyMaxActiveClusters(&count, fn, &config) != cudaSuccess || count <= 0) {
    cudaGetLastError();  // a failed query leaves no sticky error behind
    count = 16;
  }
  known[key] = count;
  return count;
}
}  // namespace

extern "C" int cb_kv_deviation_select_workspace_size(int64_t* bytes) {
  CB_REQUIRE(bytes != nullptr, "null output");
  *bytes = static_cast<int64_t>(sizeof(FusedWorkspace));
  return CB_OK;
}

extern "C" int cb_kv_deviation_select(const void* fresh, int64_t fresh_row_stride, const void* cached,
                                      int64_t cached_row_stride, int64_t cached_rows,
                                      const int64_t* abs_index, int64_t abs_offset,
                                      int64_t num_tokens, int64_t width, int dtype,
                                      const uint8_t* base_mask, int64_t k, float* scores,
                                      int64_t* out_index, int64_t out_capacity, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  CB_BIND(stream, scores);
  const int esize = dtype_bytes(dtype);
  CB_REQUIRE(esize > 0, "unsupported dtype %d", dtype);
  CB_REQUIRE(num_tokens >= 0 && width > 0 && width < (int64_t(1) << 24), "bad shape");
  CB_REQUIRE(k >= 0 && k <= num_tokens && out_capacity >= 0, "bad n/k");
  if (num_tokens == 0) return CB_OK;
  CB_REQUIRE(fresh && cached && scores && base_mask && out_index, "null pointer argument");
  CB_REQUIRE(cached_rows >= 0, "negative cached_rows");
  const uint64_t acc = reinterpret_cast<uint64_t>(fresh) | reinterpret_cast<uint64_t>(cached) |
                       (uint64_t)fresh_row_stride | (uint64_t)cached_row_stride |
                       (uint64_t)(width * esize);
  const bool vec = vector_bytes(acc) >= 16;
  const bool fits = num_tokens <= (int64_t)kClusterCtas * kFusedMaxSlice;
  if (!vec || !fits || workspace == nullptr) {
    // unaligned rows or more scores than one cluster holds: the two launches
    int rc = cb_kv_deviation(fresh, fresh_row_stride, cached, cached_row_stride, cached_rows, abs_index,
                             abs_offset, num_tokens, width, dtype, scores, stream);
    if (rc != CB_OK) return rc;
    return cb_select_topk(scores, base_mask, num_tokens, k, out_index, out_capacity, stream);
  }
  CB_REQUIRE(workspace_bytes >= (int64_t)sizeof(FusedWorkspace), "workspace too small: %lld < %zu bytes",
             (long long)workspace_bytes, sizeof(FusedWorkspace));
  CB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "workspace must be 16-byte aligned");
  const int64_t units = width * esize / 16;
  int units_log2 = 0;
  while ((int64_t(1) << units_log2) < units) ++units_log2;
  const bool small = units <= 32 && (int64_t(1) << units_log2) == units;
  const int slice = static_cast<int>((num_tokens + kClusterCtas - 1) / kClusterCtas);
  const size_t dyn = ((size_t)slice * 5 + 15) / 16 * 16;
  // clusters: as many as the GPU runs at once (one 1024-thread CTA per SM,
  // eight SMs of one GPC per cluster), fewer for short inputs
  {
    const void* fns[3][2] = {
        {(const void*)deviation_select_kernel<__nv_bfloat16, false>,
         (const void*)deviation_select_kernel<__nv_bfloat16, true>},
        {(const void*)deviation_select_kernel<__half, false>, (const void*)deviation_select_kernel<__half, true>},
        {(const void*)deviation_select_kernel<float, false>, (const void*)deviation_select_kernel<float, true>}};
    const int row = dtype == CB_DTYPE_BF16 ? 0 : (dtype == CB_DTYPE_FP16 ? 1 : 2);
    const int rc0 = ensure_dynamic_smem(fns[row][small ? 1 : 0], dyn);
    if (rc0 != CB_OK) return rc0;
  }
  int clusters = resident_clusters(small, dtype, dyn);
  const int64_t by_work = (num_tokens + 8 * 32 * 4 - 1) / (8 * 32 * 4);
  if (by_work < clusters) clusters = static_cast<int>(by_work < 1 ? 1 : by_work);
  const DevArgs args{static_cast<const char*>(fresh), fresh_row_stride, static_cast<const char*>(cached),
                     cached_row_stride, cached_rows, abs_index, abs_offset, num_tokens};
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(clusters * kClusterCtas, 1, 1);
  config.blockDim = dim3(kSelThreads, 1, 1);
  config.dynamicSmemBytes = dyn;
  config.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  const int wl = small ? units_log2 : static_cast<int>(width);
  auto* ws = static_cast<FusedWorkspace*>(workspace);
  cudaError_t e = cudaSuccess;
  int rc = CB_OK;
#define CB_FUSED_LAUNCH(T)                                                                       \
  do {                                                                                          \
    const void* fn = small ? reinterpret_cast<const void*>(deviation_select_kernel<T, true>)     \
                           : reinterpret_cast<const void*>(deviation_select_kernel<T, false>);   \
    rc = ensure_dynamic_smem(fn, dyn);                                                          \
    if (rc != CB_OK) return rc;                                                                 \
    e = small ? cudaLaunchKernelEx(&config, deviation_select_kernel<T, true>, args, wl, base_mask, \
                                   k, scores, out_index, out_capacity, slice, ws)               \
              : cudaLaunchKernelEx(&config, deviation_select_kernel<T, false>, args, wl, base_mask,\
                                   k, scores, out_index, out_capacity, slice, ws);              \
  } while (0)
  switch (dtype) {
    case CB_DTYPE_BF16:
      CB_FUSED_LAUNCH(__nv_bfloat16);
      break;
    case CB_DTYPE_FP16:
      CB_FUSED_LAUNCH(__half);
      break;
    default:
      CB_FUSED_LAUNCH(float);
      break;
  }
#undef CB_FUSED_LAUNCH
  if (e != cudaSuccess) {
    set_error("cb_kv_deviation_select cluster launch failed: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return launch_status("cb_kv_deviation_select");
}

// ---- peer exchange buffers (CUDA IPC) and the TP select ----------------------
namespace {
int64_t peer_row_capacity(int64_t n) { return (n + 3) / 4 * 4; }
int64_t peer_buffer_bytes(int world, int64_t capacity) {
  return peer_flags_offset(world, capacity) + (int64_t)(kMaxPeers + 1) * kClusterCtas * 4;
}
// Makes `device` current for this library's runtime on the calling thread.
int use_device(int device, const char* name) {
  clear_error();
  const cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_error("%s: cudaSetDevice(%d): %s", name, device, cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}
}  // namespace

extern "C" int cb_peer_select_buffer_size(int world, int64_t max_tokens, int64_t* bytes) {
  CB_REQUIRE(bytes != nullptr, "null output");
  CB_REQUIRE(world >= 1 && world <= kMaxPeers, "world size %d outside [1, %d]", world, kMaxPeers);
  CB_REQUIRE(max_tokens >= 0 && max_tokens <= (int64_t)kClusterCtas * kMaxSlice,
             "max_tokens %lld outside [0, %lld]", (long long)max_tokens,
             (long long)((int64_t)kClusterCtas * kMaxSlice));
  *bytes = peer_buffer_bytes(world, peer_row_capacity(max_tokens));
  return CB_OK;
}

extern "C" int cb_peer_buffer_create(int device, int64_t bytes, void** buffer, void* ipc_handle) {
  CB_REQUIRE(bytes > 0 && buffer != nullptr, "bad buffer request");
  const int rc = use_device(device, "cb_peer_buffer_create");
  if (rc != CB_OK) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess && ipc_handle != nullptr) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    set_error("cb_peer_buffer_create: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  *buffer = p;
  return CB_OK;
}

extern "C" int cb_peer_buffer_open(int device, const void* ipc_handle, void** buffer) {
  CB_REQUIRE(ipc_handle != nullptr && buffer != nullptr, "null argument");
  const int rc = use_device(device, "cb_peer_buffer_open");
  if (rc != CB_OK) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("cb_peer_buffer_open: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  *buffer = p;
  return CB_OK;
}

extern "C" int cb_peer_buffer_close(int device, void* buffer) {
  CB_REQUIRE(buffer != nullptr, "null buffer");
  const int rc = use_device(device, "cb_peer_buffer_close");
  if (rc != CB_OK) return rc;
  const cudaError_t e = cudaIpcCloseMemHandle(buffer);
  if (e != cudaSuccess) {
    set_error("cb_peer_buffer_close: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

extern "C" int cb_peer_buffer_destroy(int device, void* buffer) {
  CB_REQUIRE(buffer != nullptr, "null buffer");
  const int rc = use_device(device, "cb_peer_buffer_destroy");
  if (rc != CB_OK) return rc;
  const cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) {
    set_error("cb_peer_buffer_destroy: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

extern "C" int cb_peer_buffer_reset(void* buffer, int world, int64_t max_tokens, void* stream) {
  CB_REQUIRE(buffer != nullptr, "null buffer");
  CB_REQUIRE(world >= 1 && world <= kMaxPeers && max_tokens >= 0, "bad world / max_tokens");
  CB_BIND(stream, buffer);
  // the whole buffer: the counters restart at call 1, so no word of an earlier
  // call 1 or 2 may remain in the receive area
  const int64_t bytes = peer_buffer_bytes(world, peer_row_capacity(max_tokens));
  const cudaError_t e = cudaMemsetAsync(buffer, 0, static_cast<size_t>(bytes),
                                        reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("cb_peer_buffer_reset: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}

namespace {
int launch_select_peer(const float* partial, const uint8_t* base_mask, int64_t n, int64_t k,
                       int64_t* out_index, int64_t out_capacity, const uint64_t* buffers, int rank,
                       int world, int emulated, int64_t max_tokens, int protocol, float* summed,
                       int32_t* device_error, void* stream, const char* name) {
  clear_error();
  CB_REQUIRE(protocol == 0 || protocol == 1, "protocol %d is neither 0 (flags) nor 1 (low latency)", protocol);
  CB_REQUIRE(world >= 1 && world <= kMaxPeers, "world size %d outside [1, %d]", world, kMaxPeers);
  CB_REQUIRE(emulated || (rank >= 0 && rank < world), "rank %d outside [0, %d)", rank, world);
  CB_REQUIRE(buffers != nullptr && buffers[emulated ? 0 : rank] != 0, "null buffer table or own buffer");
  // this rank's own exchange buffer names the device (the scores may be empty)
  CB_BIND(stream, reinterpret_cast<const void*>(buffers[emulated ? 0 : rank]));
  CB_REQUIRE(n >= 0 && n <= max_tokens && max_tokens <= (int64_t)kClusterCtas * kMaxSlice,
             "n %lld outside [0, max_tokens %lld]", (long long)n, (long long)max_tokens);
  CB_REQUIRE(k >= 0 && k <= n && out_capacity >= 0, "bad n/k");
  CB_REQUIRE(n == 0 || (partial && base_mask), "null score or mask pointer");
  CB_REQUIRE(out_capacity == 0 || out_index, "null output pointer");
  PeerArgs args = {};
  for (int r = 0; r < world; ++r) {
    CB_REQUIRE(buffers[r] != 0 && (buffers[r] & 255) == 0, "exchange buffer %d null or unaligned", r);
    args.base[r] = buffers[r];
  }
  args.rank = emulated ? 0 : rank;
  args.world = world;
  args.emulated = emulated;
  args.low_latency = protocol;
  args.capacity = peer_row_capacity(max_tokens);
  args.flags_offset = peer_flags_offset(world, args.capacity);
  // every call exchanges, also with n == 0: the ranks' call counts stay in step
  const int slice = static_cast<int>(peer_row_capacity((n + kClusterCtas - 1) / kClusterCtas));
  const size_t dyn = ((size_t)(slice > 0 ? slice : 4) * 5 + 15) / 16 * 16;
  const int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(select_peer_kernel), dyn);
  if (rc != CB_OK) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3((emulated ? world : 1) * kClusterCtas, 1, 1);
  config.blockDim = dim3(kSelThreads, 1, 1);
  config.dynamicSmemBytes = dyn;
  config.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  config.attrs = attr;
  config.numAttrs = emulated ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&config, select_peer_kernel, partial, base_mask, n, k, out_index,
                                           out_capacity, slice > 0 ? slice : 4, args, summed, device_error);
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", name, cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return launch_status(name);
}
}  // namespace

extern "C" int cb_select_topk_peer(const float* partial, const uint8_t* base_mask, int64_t n, int64_t k,
                                   int64_t* out_index, int64_t out_capacity, const uint64_t* buffers,
                                   int rank, int world, int64_t max_tokens, int protocol, float* summed,
                                   int32_t* device_error, void* stream) {
  return launch_select_peer(partial, base_mask, n, k, out_index, out_capacity, buffers, rank, world, 0,
                            max_tokens, protocol, summed, device_error, stream, "cb_select_topk_peer");
}

extern "C" int cb_select_topk_peer_all_ranks(const float* partial, const uint8_t* base_mask, int64_t n,
                                             int64_t k, int64_t* out_index, int64_t out_capacity,
                                             const uint64_t* buffers, int world, int64_t max_tokens,
                                             int protocol, float* summed, int32_t* device_error,
                                             void* stream) {
  return launch_select_peer(partial, base_mask, n, k, out_index, out_capacity, buffers, 0, world, 1,
                            max_tokens, protocol, summed, device_error, stream,
                            "cb_select_topk_peer_all_ranks");
}
