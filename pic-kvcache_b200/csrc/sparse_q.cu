// K4: Sparse-Q attention-mass scorer on the 5th-generation tensor cores.
//
// Semantics: Qwen3BlendExecutor._sparse_q_scores (cacheblend_vllm/ascend.py:638-711).
// For every KV head h, group g and sparse query q at position pos_q, and every key
// k <= pos_q:   s = round_T(q . k) * scale   (T = bf16/fp16: the matmul output dtype)
//               p = softmax_k(s)             (fp32)
//               mass[k] += p
// summed over heads, groups and queries.  Keys beyond pos_q are masked (their
// exp is exactly 0 in the reference).
//
// Layout: rows = (query, group) pairs of one KV head, r = qi * groups + g, in
// 128-row tiles; keys in 128-key tiles.  Two passes over the causal tiles:
//   pass 1  S  = Q K^T in TMEM (lane = row): per-row online max/sum in the log2
//           domain -> lse2[h][r] = m + log2(l), stored negated (workspace)
//   pass 2  S' = K Q^T in TMEM (lane = key): each thread owns one key and sums
//           exp2(round_T(s') * scale*log2e - lse2[row]) over the rows of every
//           query tile -> one fp32 store per key, no atomics.
// Each CTA (persistent, one per SM, work dealt serpentine) is warp-specialized:
// warp 0 issues TMA tensor loads (128x64 boxes, SWIZZLE_128B, no cluster
// features), warp 1 lane 0 issues tcgen05.mma (M=128, N=128, K=16 x 8) into one
// of four TMEM accumulators, warp 2 owns the TMEM allocation, warps 4-19 are
// four softmax / accumulation warpgroups taking tiles round robin, reading
// TMEM with tcgen05.ld and computing in paired fp32 (one exp2 per score, on the
// MUFU pipe by default; the issue slots and dependency latency of this
// per-score work bound both passes).  Every mbarrier wait is
// bounded (2 s); a wait that runs out records a code in *device_error, the CTA
// drains its MMAs and TMA loads, frees TMEM and returns.
#include <mutex>
#include <type_traits>

#include "cb_common.cuh"
#include "cb_context_cache.h"
#include "cb_tcgen05.cuh"

namespace cb {
namespace sq {
using namespace ::cb::tc;

constexpr int kHead = 128;            // head_size handled by the kernels (elements)
constexpr int kStages = 3;            // streamed-operand ring
constexpr int kSmemQTiles = 4096;     // pass 2 keeps query-tile bounds in smem up to this many
constexpr int kSideSlots = 8;         // pass 2: ring of per-tile lse / position rows (1 KiB each)
// warps: 0 TMA producer, 1 MMA issuer, 2 TMEM owner, 3 spare, 4-19 four
// epilogue warpgroups taking tiles round robin (four warps per SM sub-partition
// keep the exp2 pipe fed while others wait on their TMEM loads or dependency
// chains; measured 2.4 % faster than three at config 3, 96 registers, no spills).
#ifndef CB_SQ_EPILOGUE_GROUPS
#define CB_SQ_EPILOGUE_GROUPS 4
#endif
constexpr int kEpilogueGroups = CB_SQ_EPILOGUE_GROUPS;
// Five groups (80 registers) did not complete: their bounded waits gave up
// with code 3 on the B200, so only the two measured counts are accepted.
static_assert(kEpilogueGroups == 3 || kEpilogueGroups == 4, "3 or 4 epilogue warpgroups");
constexpr int kThreads = 128 + 128 * kEpilogueGroups;
constexpr int kTmemBufs = 4;          // four 128-column fp32 accumulators
constexpr uint32_t kTmemCols = 512;

// Which score pairs take the FMA-pipe exp2 instead of the MUFU one: bit p of
// the mask (p = pair index mod 16 inside a thread's 32- or 64-score batch).
// The MUFU unit does 16 exp2 per SM per clock against 128 FMA-pipe lanes, so
// moving a share of the exp2s to the polynomial balances the two pipes.
#ifndef CB_SQ_POLY_PASS1
#define CB_SQ_POLY_PASS1 0x0000u
#endif
#ifndef CB_SQ_POLY_PASS2
#define CB_SQ_POLY_PASS2 0x0000u
#endif
constexpr uint32_t kPolyPass1 = CB_SQ_POLY_PASS1;
constexpr uint32_t kPolyPass2 = CB_SQ_POLY_PASS2;

// 2^y for two scores on the FMA pipe.  Cody-Waite style split y = j + f with
// j = rint(y), |f| <= 1/2, by adding and subtracting 1.5 * 2^23 (the sum's low
// mantissa bits then hold j); 2^f by the degree-3 polynomial of least maximum
// relative error on [-1/2, 1/2] (7.5e-5; coefficients from a Remez exchange,
// exp2_poly_fit.py beside this file); 2^j added into the exponent field.  y is
// clamped to -126 first: then j >= -126 and, since p(f) >= 2^-1/2, the biased
// exponent 126 + j of the result cannot borrow into the sign bit (at -127 and
// p(0) < 1 it would, giving NaN).  Within 7.5e-5 relative of 2^y for y >= -125;
// non-negative and below 2^-124 for smaller y (where the MUFU ex2.ftz returns
// 0 or nearly so).  Both passes only produce y <= 0 (up to one rounding).
constexpr float kExp2Round = 12582912.0f;  // 1.5 * 2^23
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;

__device__ __forceinline__ float2 exp2_poly(float2 y) {
  y.x = fmaxf(y.x, -126.0f);
  y.y = fmaxf(y.y, -126.0f);
  const float2 t = __fadd2_rn(y, make_float2(kExp2Round, kExp2Round));
  const float2 j = __fadd2_rn(t, make_float2(-kExp2Round, -kExp2Round));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), y);  // exact: y - j
  float2 p = __ffma2_rn(f, make_float2(kExp2C3, kExp2C3), make_float2(kExp2C2, kExp2C2));
  p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
  p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// 2^y of a pair, on the FMA pipe when `poly`, else on the MUFU.
__device__ __forceinline__ float2 exp2_pair(float2 y, bool poly) {
  return poly ? exp2_poly(y) : make_float2(ex2(y.x), ex2(y.y));
}

// Two fp32 accumulator values rounded (nearest even) to the 16-bit matmul
// output type T with one packed cvt; low half = lo.
template <typename T>
__device__ __forceinline__ uint32_t pack_round(uint32_t lo_bits, uint32_t hi_bits);
template <>
__device__ __forceinline__ uint32_t pack_round<__nv_bfloat16>(uint32_t lo_bits, uint32_t hi_bits) {
  uint32_t packed;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "r"(hi_bits), "r"(lo_bits));
  return packed;
}
template <>
__device__ __forceinline__ uint32_t pack_round<__half>(uint32_t lo_bits, uint32_t hi_bits) {
  uint32_t packed;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(packed) : "r"(hi_bits), "r"(lo_bits));
  return packed;
}

// The pair widened back to fp32.
template <typename T>
__device__ __forceinline__ float2 unpack(uint32_t packed);
template <>
__device__ __forceinline__ float2 unpack<__nv_bfloat16>(uint32_t packed) {
  return make_float2(__uint_as_float(packed << 16), __uint_as_float(packed & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack<__half>(uint32_t packed) {
  return __half22float2(*reinterpret_cast<const __half2*>(&packed));
}

// Elementwise max of two packed pairs (one instruction for two scores).
template <typename T>
__device__ __forceinline__ uint32_t pair_max(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t pair_max<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <>
__device__ __forceinline__ uint32_t pair_max<__half>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// -inf in T's encoding, in the low half of a packed pair.
template <typename T>
__device__ __forceinline__ constexpr uint32_t neg_inf_half() {
  return std::is_same<T, __nv_bfloat16>::value ? 0xff80u : 0xfc00u;
}

// Named barrier over the epilogue warpgroups.
__device__ __forceinline__ void epilogue_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(128 * kEpilogueGroups) : "memory");
}

// Instruction descriptor: D f32 (bits 4-5 = 1), A and B bf16 (1) or f16 (0)
// in bits 7-9 / 10-12, both K-major (bits 15, 16 = 0), N>>3 in bits 17-22,
// M>>4 in bits 24-28; M = N = 128.
template <typename T>
__host__ __device__ constexpr uint32_t instr_desc() {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(kTile >> 3) << 17) |
         ((uint32_t)(kTile >> 4) << 24);
}

struct Shared {
  // operand buffers live in dynamic shared memory (1024-B aligned), barriers here
  uint64_t a_full[2], a_empty[2];
  uint64_t b_full[kStages], b_empty[kStages];
  uint64_t t_full[kTmemBufs], t_empty[kTmemBufs];
  uint64_t side_full[kSideSlots], side_empty[kSideSlots];  // pass 2 lse / position ring
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float merge[kEpilogueGroups - 1][2][kTile];  // other warpgroups' row stats / key sums
};

struct Common {
  int num_kv_heads;
  int groups;
  int rows_pad;        // padded rows per KV head
  int q_tiles;         // rows_pad / 128
  int k_tiles;         // ceil(num_keys / 128)
  int64_t num_keys;
  float scale_log2;    // scale * log2(e)
  const int32_t* row_pos;   // [rows_pad]: position of each row, -1 for padding
  const int32_t* tile_max;  // [q_tiles]
  const int32_t* tile_min;  // [q_tiles]
  float* lse;               // [num_kv_heads][rows_pad]: -(log2-sum-exp) per row (pass 1 out, pass 2 in)
  float* scores;            // [num_keys] (pass 2 out)
  int32_t* error;
};

__device__ __forceinline__ void report(const Common& c, Shared& sh, int code) {
  if (c.error != nullptr) atomicCAS(c.error, 0, code);
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
}

__device__ __forceinline__ bool aborted(Shared& sh) {
  return *reinterpret_cast<volatile int*>(&sh.abort) != 0;
}

// Setup shared by both passes: barriers + TMEM allocation.
__device__ __forceinline__ void setup(Shared& sh, int warp, int a_empty_count, int b_empty_count) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sh.a_full[i], 1);
      mbar_init(&sh.a_empty[i], a_empty_count);
    }
    for (int i = 0; i < kTmemBufs; ++i) {
      mbar_init(&sh.t_full[i], 1);
      mbar_init(&sh.t_empty[i], 4);  // one arrive per warp of the owning warpgroup
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.b_full[s], 1);
      mbar_init(&sh.b_empty[s], b_empty_count);
    }
    for (int q = 0; q < kSideSlots; ++q) {
      mbar_init(&sh.side_full[q], 1);
      mbar_init(&sh.side_empty[q], 4);  // the four warps of the warpgroup that read the slot
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sh.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

__device__ __forceinline__ void teardown(Shared& sh, int warp) {
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// k-th work item of this CTA.  Items are numbered in decreasing cost (pass 1:
// later query tiles see more keys; pass 2: earlier key tiles are seen by more
// queries), so a serpentine deal -- each round in the opposite direction --
// balances the per-CTA totals; plain round robin left SMs idle 18 % of the time.
// Once an item is out of range every later one is too.
__device__ __forceinline__ int cta_item(int k) {
  const int g = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  return k * g + ((k & 1) ? g - 1 - c : c);
}

// MMA issuer drain: wait until every MMA this thread issued has completed.
__device__ __forceinline__ void drain_mma(Shared& sh) {
  umma_commit(&sh.drain);
  wait1(&sh.drain, 0);
}

// ============================================================ pass 1: row LSE
// items: (h, qt) with qt descending (later queries see more keys).
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    lse_pass_kernel(const __grid_constant__ CUtensorMap q_map,
                    const __grid_constant__ CUtensorMap k_map, Common c) {
  extern __shared__ __align__(1024) unsigned char dyn[];
  __shared__ Shared sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dyn) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* a_buf = base;                   // 2 x Q tiles
  unsigned char* b_buf = base + 2 * kTileBytes;  // kStages x K tiles
  setup(sh, warp, 1, 1);
  const int items = c.num_kv_heads * c.q_tiles;

  if (warp == 0) {
    if (lane == 0) {
      int t = 0, it = 0;
      int armed[kStages];
      for (int s = 0; s < kStages; ++s) armed[s] = -1;
      int a_armed[2] = {-1, -1};
      for (int k = 0, item = cta_item(0); item < items && !aborted(sh); item = cta_item(++k), ++it) {
        const int qt = c.q_tiles - 1 - item / c.num_kv_heads;
        const int h = item % c.num_kv_heads;
        const int ab = it & 1;
        if (!wait1(&sh.a_empty[ab], ((it >> 1) & 1) ^ 1)) { report(c, sh, 1); break; }
        mbar_expect_tx(&sh.a_full[ab], kTileBytes);
        tma_load_3d(a_buf + ab * kTileBytes, &q_map, &sh.a_full[ab], 0, qt * kTile, h);
        tma_load_3d(a_buf + ab * kTileBytes + kHalfBytes, &q_map, &sh.a_full[ab], 64, qt * kTile, h);
        a_armed[ab] = (it >> 1) & 1;
        const int kt_end = min(c.tile_max[qt] / kTile, c.k_tiles - 1);  // tile_max >= 0 here
        for (int kt = 0; kt <= kt_end; ++kt, ++t) {
          const int s = t % kStages;
          if (!wait1(&sh.b_empty[s], ((t / kStages) & 1) ^ 1)) { report(c, sh, 1); break; }
          mbar_expect_tx(&sh.b_full[s], kTileBytes);
          tma_load_3d(b_buf + s * kTileBytes, &k_map, &sh.b_full[s], 0, h, kt * kTile);
          tma_load_3d(b_buf + s * kTileBytes + kHalfBytes, &k_map, &sh.b_full[s], 64, h, kt * kTile);
          armed[s] = (t / kStages) & 1;
        }
      }
      // drain: every armed load has landed before the CTA may exit
      for (int s = 0; s < kStages; ++s)
        if (armed[s] >= 0) wait1(&sh.b_full[s], armed[s]);
      for (int i = 0; i < 2; ++i)
        if (a_armed[i] >= 0) wait1(&sh.a_full[i], a_armed[i]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc<T>();
      const uint32_t a_addr = smem_u32(a_buf);
      const uint32_t b_addr = smem_u32(b_buf);
      int t = 0, it = 0;
      for (int k = 0, item = cta_item(0); item < items && !aborted(sh); item = cta_item(++k), ++it) {
        const int qt = c.q_tiles - 1 - item / c.num_kv_heads;
        const int ab = it & 1;
        if (!wait1(&sh.a_full[ab], (it >> 1) & 1)) { report(c, sh, 2); break; }
        const int kt_end = min(c.tile_max[qt] / kTile, c.k_tiles - 1);
        bool ok = true;
        for (int kt = 0; kt <= kt_end; ++kt, ++t) {
          const int s = t % kStages;
          const int tb = t & (kTmemBufs - 1);
          if (!wait1(&sh.b_full[s], (t / kStages) & 1) ||
              !wait1(&sh.t_empty[tb], ((t / kTmemBufs) & 1) ^ 1)) {
            report(c, sh, 2);
            ok = false;
            break;
          }
          tc_fence_after();
          umma_k128(sh.tmem_base + tb * kTile, a_addr + ab * kTileBytes, b_addr + s * kTileBytes,
                    idesc, false);
          umma_commit(&sh.b_empty[s]);
          umma_commit(&sh.t_full[tb]);
        }
        umma_commit(&sh.a_empty[ab]);
        if (!ok) break;
      }
      drain_mma(sh);
    }
  } else if (warp >= 4) {
    const int wg = (warp - 4) >> 2;       // epilogue warpgroup: takes tiles with t % 3 == wg
    const int ew = warp & 3;              // TMEM lanes 32*ew .. +31
    const int row_in_tile = ew * 32 + lane;
    int t0 = 0;
    bool ok = true;
    for (int k = 0, item = cta_item(0); item < items; item = cta_item(++k)) {
      const int qt = c.q_tiles - 1 - item / c.num_kv_heads;
      const int h = item % c.num_kv_heads;
      const int r = qt * kTile + row_in_tile;
      const int pos = c.row_pos[r];
      const int kt_end = min(c.tile_max[qt] / kTile, c.k_tiles - 1);
      float m = -INFINITY, l = 0.0f;  // log2-domain running max and sum of this row
      for (int kt = 0; kt <= kt_end && ok; ++kt) {
        const int t = t0 + kt;
        if (t % kEpilogueGroups != wg) continue;
        const int tb = t & (kTmemBufs - 1);
        if (!wait_warp(&sh.t_full[tb], (t / kTmemBufs) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t addr = sh.tmem_base + tb * kTile + (static_cast<uint32_t>(ew * 32) << 16);
        const int valid = min(max(pos - kt * kTile + 1, 0), kTile);  // keys <= pos
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v[2][32];
          tmem_ld32(addr + half * 64, v[0]);
          tmem_ld32(addr + half * 64 + 32, v[1]);
          tmem_wait_ld();
          if (half == 1) {  // the accumulator goes back to the MMA
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.t_empty[tb]);
          }
          const int lim = valid - half * 64;  // valid columns in this half
          if (lim <= 0) continue;
          uint32_t pk[32];  // the 64 rounded logits, packed in pairs (low half = even column)
#pragma unroll
          for (int j = 0; j < 32; ++j)
            pk[j] = pack_round<T>(v[j >> 4][(2 * j) & 31], v[j >> 4][(2 * j + 1) & 31]);
          if (lim < 64) {  // keys past the row's position: -inf
            constexpr uint32_t ninf = neg_inf_half<T>();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (2 * j >= lim) pk[j] = ninf | (ninf << 16);
              else if (2 * j + 1 >= lim) pk[j] = (pk[j] & 0xffffu) | (ninf << 16);
            }
          }
          // row max: four packed chains, one max per two scores
          uint32_t mk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) mk[i] = pk[i];
#pragma unroll
          for (int j = 4; j < 32; ++j) mk[j & 3] = pair_max<T>(mk[j & 3], pk[j]);
          const float2 mm = unpack<T>(pair_max<T>(pair_max<T>(mk[0], mk[1]), pair_max<T>(mk[2], mk[3])));
          const float cmax = fmaxf(mm.x, mm.y);
          const float m_new = fmaxf(m, cmax * c.scale_log2);  // scale > 0: max commutes
          // paired fp32 FMA / add: one instruction per two scores
          const float2 scale2 = make_float2(c.scale_log2, c.scale_log2);
          const float2 shift2 = make_float2(-m_new, -m_new);
          float2 sm[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) sm[i] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float2 y = __ffma2_rn(unpack<T>(pk[j]), scale2, shift2);
            sm[j & 3] = __fadd2_rn(sm[j & 3], exp2_pair(y, (kPolyPass1 >> (j & 15)) & 1u));
          }
          const float2 s01 = __fadd2_rn(sm[0], sm[1]);
          const float2 s23 = __fadd2_rn(sm[2], sm[3]);
          const float2 s03 = __fadd2_rn(s01, s23);
          const float part = s03.x + s03.y;
          l = l * ex2(m - m_new) + part;
          m = m_new;
        }
      }
      t0 += kt_end + 1;
      // merge the warpgroups' partial statistics of this row.  After an error
      // every warpgroup still passes both barriers (without waiting on the
      // pipeline) so none blocks in bar.sync.
      if (wg > 0) {
        sh.merge[wg - 1][0][row_in_tile] = m;
        sh.merge[wg - 1][1][row_in_tile] = l;
      }
      epilogue_sync();
      if (wg == 0) {
        float ms[kEpilogueGroups], ls[kEpilogueGroups];
        ms[0] = m;
        ls[0] = l;
        float mx = m;
#pragma unroll
        for (int g = 1; g < kEpilogueGroups; ++g) {
          ms[g] = sh.merge[g - 1][0][row_in_tile];
          ls[g] = sh.merge[g - 1][1][row_in_tile];
          mx = fmaxf(mx, ms[g]);
        }
        float total = 0.0f;
#pragma unroll
        for (int g = 0; g < kEpilogueGroups; ++g)
          if (ls[g] > 0.0f) total += ls[g] * ex2(ms[g] - mx);
        // stored negated: pass 2 adds it in a paired FMA
        c.lse[(int64_t)h * c.rows_pad + r] = total > 0.0f ? -(mx + lg2(total)) : -INFINITY;
      }
      epilogue_sync();
    }
    if (!ok && lane == 0) report(c, sh, 3);
  }
  teardown(sh, warp);
}

// Pass 2's work on 4 * J rows of one key (this lane's): scores v[] (fp32 bits
// from TMEM), the rows' negated log2-sum-exp and positions from the side slot.
// Adds exp2(round_T(s) * scale * log2e - lse) into acc; rows past the key's
// position add 0 when the tile is not `full`.
template <typename T, int J, int N>
__device__ __forceinline__ void key_mass_rows(const uint32_t (&v)[N], const float4* nlse4,
                                              const int4* pos4, bool full, int key, float2 scale2,
                                              float2 (&acc)[4]) {
  static_assert(N == 4 * J, "four rows per step");
  if (full) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float4 l4 = nlse4[j];
      const float2 y0 = __ffma2_rn(unpack<T>(pack_round<T>(v[4 * j], v[4 * j + 1])), scale2,
                                   make_float2(l4.x, l4.y));
      const float2 y1 = __ffma2_rn(unpack<T>(pack_round<T>(v[4 * j + 2], v[4 * j + 3])), scale2,
                                   make_float2(l4.z, l4.w));
      acc[(2 * j) & 3] = __fadd2_rn(acc[(2 * j) & 3], exp2_pair(y0, (kPolyPass2 >> ((2 * j) & 15)) & 1u));
      acc[(2 * j + 1) & 3] =
          __fadd2_rn(acc[(2 * j + 1) & 3], exp2_pair(y1, (kPolyPass2 >> ((2 * j + 1) & 15)) & 1u));
    }
  } else {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float4 l4 = nlse4[j];
      const int4 p4 = pos4[j];
      const float2 y0 = __ffma2_rn(unpack<T>(pack_round<T>(v[4 * j], v[4 * j + 1])), scale2,
                                   make_float2(l4.x, l4.y));
      const float2 y1 = __ffma2_rn(unpack<T>(pack_round<T>(v[4 * j + 2], v[4 * j + 3])), scale2,
                                   make_float2(l4.z, l4.w));
      const float2 e0 = make_float2(key <= p4.x ? ex2(y0.x) : 0.0f, key <= p4.y ? ex2(y0.y) : 0.0f);
      const float2 e1 = make_float2(key <= p4.z ? ex2(y1.x) : 0.0f, key <= p4.w ? ex2(y1.y) : 0.0f);
      acc[(2 * j) & 3] = __fadd2_rn(acc[(2 * j) & 3], e0);
      acc[(2 * j + 1) & 3] = __fadd2_rn(acc[(2 * j + 1) & 3], e1);
    }
  }
}

// ============================================================ pass 2: key mass
// items: key tiles kt ascending (earlier keys are seen by more queries).
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    mass_pass_kernel(const __grid_constant__ CUtensorMap q_map,
                     const __grid_constant__ CUtensorMap k_map, Common c) {
  extern __shared__ __align__(1024) unsigned char dyn[];
  __shared__ Shared sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dyn) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* a_buf = base;                   // 2 x K tiles
  unsigned char* b_buf = base + 2 * kTileBytes;  // kStages x (Q tile)
  // per side slot: -lse[128], pos[128] of one streamed query tile.  Kept apart from the
  // query tile so that the MMA alone frees a query stage: the epilogue warpgroups
  // holding the stages until they finish would starve the loads.
  float* side = reinterpret_cast<float*>(b_buf + kStages * kTileBytes);
  // Every role scans the query tiles' position bounds for every key tile:
  // keep them in shared memory when they fit (copied before setup's barrier).
  const int* tile_max = c.tile_max;
  const int* tile_min = c.tile_min;
  if (c.q_tiles <= kSmemQTiles) {
    int* bounds = reinterpret_cast<int*>(side + kSideSlots * 2 * kTile);
    for (int i = threadIdx.x; i < c.q_tiles; i += blockDim.x) {
      bounds[i] = c.tile_max[i];
      bounds[c.q_tiles + i] = c.tile_min[i];
    }
    tile_max = bounds;
    tile_min = bounds + c.q_tiles;
  }
  setup(sh, warp, 1, 1);  // b_empty: the MMA commit
  const int items = c.k_tiles;

  if (warp == 0) {
    if (lane == 0) {
      int t = 0, it = 0;
      int armed[kStages];
      for (int s = 0; s < kStages; ++s) armed[s] = -1;
      int a_armed[2] = {-1, -1};
      int side_armed[kSideSlots];
      for (int q = 0; q < kSideSlots; ++q) side_armed[q] = -1;
      for (int k = 0, kt = cta_item(0); kt < items && !aborted(sh); kt = cta_item(++k)) {
        for (int h = 0; h < c.num_kv_heads && !aborted(sh); ++h, ++it) {
          const int ab = it & 1;
          if (!wait1(&sh.a_empty[ab], ((it >> 1) & 1) ^ 1)) { report(c, sh, 1); break; }
          mbar_expect_tx(&sh.a_full[ab], kTileBytes);
          tma_load_3d(a_buf + ab * kTileBytes, &k_map, &sh.a_full[ab], 0, h, kt * kTile);
          tma_load_3d(a_buf + ab * kTileBytes + kHalfBytes, &k_map, &sh.a_full[ab], 64, h, kt * kTile);
          a_armed[ab] = (it >> 1) & 1;
          for (int qt = 0; qt < c.q_tiles; ++qt) {
            if (tile_max[qt] < kt * kTile) continue;  // no row of this tile sees these keys
            const int s = t % kStages;
            const int q = t % kSideSlots;
            if (!wait1(&sh.b_empty[s], ((t / kStages) & 1) ^ 1) ||
                !wait1(&sh.side_empty[q], ((t / kSideSlots) & 1) ^ 1)) {
              report(c, sh, 1);
              break;
            }
            mbar_expect_tx(&sh.b_full[s], kTileBytes);
            tma_load_3d(b_buf + s * kTileBytes, &q_map, &sh.b_full[s], 0, qt * kTile, h);
            tma_load_3d(b_buf + s * kTileBytes + kHalfBytes, &q_map, &sh.b_full[s], 64, qt * kTile, h);
            armed[s] = (t / kStages) & 1;
            mbar_expect_tx(&sh.side_full[q], 2 * kTile * 4);
            bulk_load(side + q * 2 * kTile, c.lse + (int64_t)h * c.rows_pad + qt * kTile, kTile * 4,
                      &sh.side_full[q]);
            bulk_load(side + q * 2 * kTile + kTile, c.row_pos + qt * kTile, kTile * 4, &sh.side_full[q]);
            side_armed[q] = (t / kSideSlots) & 1;
            ++t;
          }
        }
      }
      for (int s = 0; s < kStages; ++s)
        if (armed[s] >= 0) wait1(&sh.b_full[s], armed[s]);
      for (int q = 0; q < kSideSlots; ++q)
        if (side_armed[q] >= 0) wait1(&sh.side_full[q], side_armed[q]);
      for (int i = 0; i < 2; ++i)
        if (a_armed[i] >= 0) wait1(&sh.a_full[i], a_armed[i]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = instr_desc<T>();
      const uint32_t a_addr = smem_u32(a_buf);
      const uint32_t b_addr = smem_u32(b_buf);
      int t = 0, it = 0;
      bool ok = true;
      for (int k = 0, kt = cta_item(0); kt < items && ok && !aborted(sh); kt = cta_item(++k)) {
        for (int h = 0; h < c.num_kv_heads && ok; ++h, ++it) {
          const int ab = it & 1;
          if (!wait1(&sh.a_full[ab], (it >> 1) & 1)) { report(c, sh, 2); ok = false; break; }
          for (int qt = 0; qt < c.q_tiles; ++qt) {
            if (tile_max[qt] < kt * kTile) continue;
            const int s = t % kStages;
            const int tb = t & (kTmemBufs - 1);
            if (!wait1(&sh.b_full[s], (t / kStages) & 1) ||
                !wait1(&sh.t_empty[tb], ((t / kTmemBufs) & 1) ^ 1)) {
              report(c, sh, 2);
              ok = false;
              break;
            }
            tc_fence_after();
            umma_k128(sh.tmem_base + tb * kTile, a_addr + ab * kTileBytes, b_addr + s * kTileBytes,
                      idesc, false);
            umma_commit(&sh.b_empty[s]);
            umma_commit(&sh.t_full[tb]);
            ++t;
          }
          umma_commit(&sh.a_empty[ab]);
        }
      }
      drain_mma(sh);
    }
  } else if (warp >= 4) {
    const int wg = (warp - 4) >> 2;
    const int ew = warp & 3;
    const int key_in_tile = ew * 32 + lane;
    int t = 0;
    bool ok = true;
    for (int k = 0, kt = cta_item(0); kt < items; kt = cta_item(++k)) {
      const int key = kt * kTile + key_in_tile;
      float2 acc[4];  // eight independent sums of this key's mass, in pairs
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
      const float2 scale2 = make_float2(c.scale_log2, c.scale_log2);
      for (int h = 0; h < c.num_kv_heads && ok; ++h) {
        for (int qt = 0; qt < c.q_tiles; ++qt) {
          if (tile_max[qt] < kt * kTile) continue;
          const int mine = t % kEpilogueGroups == wg;
          const int q = t % kSideSlots;
          const int tb = t & (kTmemBufs - 1);
          const uint32_t tp = (t / kTmemBufs) & 1;
          const uint32_t qp = (t / kSideSlots) & 1;
          ++t;
          if (!mine) continue;
          if (!wait_warp(&sh.side_full[q], qp) || !wait_warp(&sh.t_full[tb], tp)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t addr = sh.tmem_base + tb * kTile + (static_cast<uint32_t>(ew * 32) << 16);
          const float* nlse = side + q * 2 * kTile;  // -lse of each row
          const int* pos = reinterpret_cast<const int*>(side + q * 2 * kTile + kTile);
          const bool full = key <= tile_min[qt];  // every row of the tile sees this key
#pragma unroll
          for (int quarter = 0; quarter < 4; ++quarter) {
            uint32_t v[32];  // 32 rows of this key: one TMEM load, few live registers
            tmem_ld32(addr + quarter * 32, v);
            tmem_wait_ld();
            if (quarter == 3) {  // TMEM no longer needed: hand the accumulator back to the MMA
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&sh.t_empty[tb]);
            }
            const float4* nlse4 = reinterpret_cast<const float4*>(nlse + quarter * 32);
            const int4* pos4 = reinterpret_cast<const int4*>(pos + quarter * 32);
            key_mass_rows<T, 8>(v, nlse4, pos4, full, key, scale2, acc);
            if (quarter == 3) {  // lse / positions of this slot read: release it
              __syncwarp();
              if (lane == 0) mbar_arrive(&sh.side_empty[q]);
            }
          }
        }
      }
      const float2 a03 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
      const float mass = a03.x + a03.y;
      // merge the warpgroups' sums for this key tile (reached by every
      // warpgroup for every item, also after an error)
      if (wg > 0) sh.merge[wg - 1][0][key_in_tile] = mass;
      epilogue_sync();
      if (wg == 0 && key < c.num_keys) {
        float total = mass;
#pragma unroll
        for (int g = 1; g < kEpilogueGroups; ++g) total += sh.merge[g - 1][0][key_in_tile];
        c.scores[key] = total;
      }
      epilogue_sync();
    }
    if (!ok && lane == 0) report(c, sh, 3);
  }
  teardown(sh, warp);
}

// ============================================================ prep
// Dense per-KV-head query rows: qd[h][qi*groups+g][:] = query[rows[qi]][h*groups+g][:],
// zero rows up to rows_pad; row positions; per-tile position bounds.  A query
// row outside [0, query_tokens) or a negative position is not read: its rows
// are zero and masked (position -1, they see no key) and code 4 is recorded in
// *error.  A position past the last key sees every key, as the reference's
// mask `pos_q < key_position` does, so it is clamped to num_keys - 1.
__device__ __forceinline__ int query_position(const int64_t* rows, const int64_t* positions,
                                              int64_t qi, int64_t query_tokens, int64_t num_keys) {
  const int64_t row = rows[qi];
  const int64_t pos = positions[qi];
  if (row < 0 || row >= query_tokens || pos < 0) return -1;
  return static_cast<int>(pos < num_keys ? pos : num_keys - 1);
}

__global__ void __launch_bounds__(256) prep_kernel(const char* __restrict__ query,
                                                   int64_t query_token_stride, int64_t query_tokens,
                                                   const int64_t* __restrict__ rows,
                                                   const int64_t* __restrict__ positions,
                                                   int64_t num_queries, int64_t num_keys,
                                                   int num_kv_heads, int groups,
                                                   int rows_pad, int head_bytes, char* __restrict__ qd,
                                                   int32_t* __restrict__ row_pos,
                                                   int32_t* __restrict__ tile_max,
                                                   int32_t* __restrict__ tile_min,
                                                   int32_t* __restrict__ error) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t total = static_cast<int64_t>(num_kv_heads) * rows_pad;
  const int units = head_bytes / 16;
  for (int64_t task = warp; task < total; task += nwarps) {
    const int h = static_cast<int>(task / rows_pad);
    const int r = static_cast<int>(task - (int64_t)h * rows_pad);
    const int64_t qi = r / groups;
    const int g = r - static_cast<int>(qi) * groups;
    uint4* dst = reinterpret_cast<uint4*>(qd + task * head_bytes);
    const int pos = qi < num_queries ? query_position(rows, positions, qi, query_tokens, num_keys) : -1;
    if (pos >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(
          query + rows[qi] * query_token_stride + (int64_t)(h * groups + g) * head_bytes);
      for (int u = lane; u < units; u += 32) dst[u] = src[u];
    } else {
      for (int u = lane; u < units; u += 32) dst[u] = make_uint4(0, 0, 0, 0);
      if (qi < num_queries && h == 0 && g == 0 && lane == 0 && error != nullptr)
        atomicCAS(error, 0, 4);
    }
    if (h == 0 && lane == 0) row_pos[r] = pos;
  }
  // tile bounds: one warp per query tile
  const int q_tiles = rows_pad / kTile;
  for (int64_t qt = warp; qt < q_tiles; qt += nwarps) {
    int mx = -1, mn = 0x7fffffff;
    for (int r = lane; r < kTile; r += 32) {
      const int64_t qi = (qt * kTile + r) / groups;
      const int p = qi < num_queries ? query_position(rows, positions, qi, query_tokens, num_keys) : -1;
      mx = max(mx, p);
      mn = min(mn, p);  // a masked row (-1) makes the tile "partially visible": always masked
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    }
    if (lane == 0) {
      tile_max[qt] = mx;
      tile_min[qt] = mn;
    }
  }
}

// ---------------------------------------------------------------- host side
struct Workspace {
  size_t qd, lse, row_pos, tile_max, tile_min, total;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Workspace layout(int64_t num_queries, int64_t num_q_heads, int64_t num_kv_heads, int esize) {
  const int64_t groups = num_q_heads / num_kv_heads;
  const int64_t rows = num_queries * groups;
  const int64_t rows_pad = (rows + kTile - 1) / kTile * kTile;
  const int64_t q_tiles = rows_pad / kTile;
  Workspace w{};
  size_t off = 0;
  w.qd = off;
  off = align_up(off + (size_t)num_kv_heads * rows_pad * kHead * esize, 1024);
  w.lse = off;
  off = align_up(off + (size_t)num_kv_heads * rows_pad * 4, 1024);
  w.row_pos = off;
  off = align_up(off + (size_t)rows_pad * 4, 256);
  w.tile_max = off;
  off = align_up(off + (size_t)q_tiles * 4, 256);
  w.tile_min = off;
  off = align_up(off + (size_t)q_tiles * 4, 256);
  w.total = off;
  return w;
}

constexpr size_t kDynSmem1 = 1024 + (2 + kStages) * kTileBytes;
constexpr size_t kDynSmem2 = 1024 + (2 + kStages) * kTileBytes + kSideSlots * 2 * kTile * 4;

template <typename T>
int launch_passes(const CUtensorMap& q_map, const CUtensorMap& k_map, const Common& c,
                  cudaStream_t s) {
  const int grid1 = min(c.num_kv_heads * c.q_tiles, kSmCount);
  const int grid2 = min(c.k_tiles, kSmCount);
  int rc0 = ensure_dynamic_smem(reinterpret_cast<const void*>(lse_pass_kernel<T>), kDynSmem1);
  if (rc0 == CB_OK)
    rc0 = ensure_dynamic_smem(reinterpret_cast<const void*>(mass_pass_kernel<T>),
                              kDynSmem2 + 2 * kSmemQTiles * sizeof(int));
  if (rc0 != CB_OK) return rc0;
  lse_pass_kernel<T><<<grid1, kThreads, kDynSmem1, s>>>(q_map, k_map, c);
  int rc = launch_status("cb_sparse_q_scores (row pass)");
  if (rc != CB_OK) return rc;
  const size_t smem2 = kDynSmem2 + (c.q_tiles <= kSmemQTiles ? 2 * c.q_tiles * sizeof(int) : 0);
  mass_pass_kernel<T><<<grid2, kThreads, smem2, s>>>(q_map, k_map, c);
  return launch_status("cb_sparse_q_scores (key pass)");
}

int check_shape(int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int dtype) {
  CB_SUPPORTED(dtype == CB_DTYPE_BF16 || dtype == CB_DTYPE_FP16,
               "Sparse-Q tensor-core scorer needs bf16 or fp16 query/key");
  CB_SUPPORTED(head_size == kHead, "Sparse-Q tensor-core scorer supports head_size 128 (got %lld)",
               (long long)head_size);
  CB_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
             "query heads must be a multiple of KV heads");
  const int64_t groups = num_q_heads / num_kv_heads;
  CB_SUPPORTED(groups <= kTile && kTile % groups == 0, "query groups must divide 128");
  return CB_OK;
}

}  // namespace sq
}  // namespace cb

using namespace cb;

extern "C" int cb_sparse_q_workspace_size(int64_t num_queries, int64_t num_q_heads,
                                          int64_t num_kv_heads, int64_t head_size, int dtype,
                                          int64_t* bytes) {
  CB_REQUIRE(bytes != nullptr, "null output");
  int rc = sq::check_shape(num_q_heads, num_kv_heads, head_size, dtype);
  if (rc != CB_OK) return rc;
  CB_REQUIRE(num_queries >= 0 && num_queries < (int64_t(1) << 30) &&
                 num_queries * (num_q_heads / num_kv_heads) < (int64_t(1) << 30),
             "too many queries");
  CB_REQUIRE(num_kv_heads <= 1024, "too many KV heads");
  *bytes = static_cast<int64_t>(sq::layout(num_queries, num_q_heads, num_kv_heads, 2).total);
  return CB_OK;
}

namespace cb {
namespace sq {
// Argument checks shared by both entry points; everything a size computation
// multiplies is bounded first, so no product below can overflow.
int check_counts(int64_t num_query_tokens, int64_t num_keys, int64_t num_q_heads,
                 int64_t num_kv_heads, int64_t num_queries) {
  CB_REQUIRE(num_keys >= 0 && num_keys < (int64_t(1) << 31), "num_keys out of range");
  CB_REQUIRE(num_query_tokens >= 0, "negative query token count");
  CB_REQUIRE(num_queries >= 0 && num_queries < (int64_t(1) << 30) &&
                 num_queries * (num_q_heads / num_kv_heads) < (int64_t(1) << 30),
             "too many queries");
  CB_REQUIRE(num_kv_heads <= 1024, "too many KV heads");
  return CB_OK;
}
}  // namespace sq
}  // namespace cb

extern "C" int cb_sparse_q_scores(const void* query, int64_t query_token_stride,
                                  int64_t num_query_tokens, const void* key,
                                  int64_t key_token_stride, int64_t num_keys, int64_t num_q_heads,
                                  int64_t num_kv_heads, int64_t head_size, int dtype,
                                  const int64_t* query_rows, const int64_t* query_positions,
                                  int64_t num_queries, float scale, float* scores, void* workspace,
                                  int64_t workspace_bytes, int32_t* device_error, void* stream) {
  CB_BIND(stream, scores);
  int rc = sq::check_shape(num_q_heads, num_kv_heads, head_size, dtype);
  if (rc != CB_OK) return rc;
  rc = sq::check_counts(num_query_tokens, num_keys, num_q_heads, num_kv_heads, num_queries);
  if (rc != CB_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (num_keys == 0) return CB_OK;
  CB_REQUIRE(scores != nullptr && key != nullptr, "null pointer argument");
  if (num_queries == 0) {
    // no query sees any key: the mass is zero everywhere
    cudaError_t e = cudaMemsetAsync(scores, 0, num_keys * sizeof(float), s);
    if (e != cudaSuccess) {
      set_error("cudaMemsetAsync failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
    return CB_OK;
  }
  CB_REQUIRE(query && query_rows && query_positions && workspace, "null pointer argument");
  const int esize = 2;
  const sq::Workspace w = sq::layout(num_queries, num_q_heads, num_kv_heads, esize);
  CB_REQUIRE(workspace_bytes >= (int64_t)w.total, "workspace too small: %lld < %lld bytes",
             (long long)workspace_bytes, (long long)w.total);
  CB_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 1023) == 0, "workspace must be 1 KiB aligned");
  const uint64_t row_bytes = (uint64_t)num_kv_heads * head_size * esize;
  CB_REQUIRE(((reinterpret_cast<uintptr_t>(key) | (uint64_t)key_token_stride |
               (reinterpret_cast<uintptr_t>(query) | (uint64_t)query_token_stride)) & 15) == 0,
             "query/key rows must be 16-byte aligned");
  CB_REQUIRE(key_token_stride >= (int64_t)row_bytes, "key rows overlap");
  const int groups = static_cast<int>(num_q_heads / num_kv_heads);
  const int rows_pad = static_cast<int>((num_queries * groups + sq::kTile - 1) / sq::kTile * sq::kTile);
  char* ws = static_cast<char*>(workspace);
  sq::Common c{};
  c.num_kv_heads = static_cast<int>(num_kv_heads);
  c.groups = groups;
  c.rows_pad = rows_pad;
  c.q_tiles = rows_pad / sq::kTile;
  c.k_tiles = static_cast<int>((num_keys + sq::kTile - 1) / sq::kTile);
  c.num_keys = num_keys;
  c.scale_log2 = scale * 1.4426950408889634f;
  c.row_pos = reinterpret_cast<const int32_t*>(ws + w.row_pos);
  c.tile_max = reinterpret_cast<const int32_t*>(ws + w.tile_max);
  c.tile_min = reinterpret_cast<const int32_t*>(ws + w.tile_min);
  c.lse = reinterpret_cast<float*>(ws + w.lse);
  c.scores = scores;
  c.error = device_error;

  {
    const int64_t warps = num_kv_heads * rows_pad;
    const int64_t blocks = (warps + 7) / 8;
    const int grid = static_cast<int>(blocks < kSmCount * 8 ? blocks : kSmCount * 8);
    sq::prep_kernel<<<grid, 256, 0, s>>>(
        static_cast<const char*>(query), query_token_stride, num_query_tokens, query_rows,
        query_positions, num_queries, num_keys, c.num_kv_heads, groups, rows_pad,
        static_cast<int>(head_size * esize), ws + w.qd, reinterpret_cast<int32_t*>(ws + w.row_pos),
        reinterpret_cast<int32_t*>(ws + w.tile_max), reinterpret_cast<int32_t*>(ws + w.tile_min),
        device_error);
    rc = launch_status("cb_sparse_q_scores (prep)");
    if (rc != CB_OK) return rc;
  }
  sq::EncodeTiled encode;
  rc = sq::get_encoder(&encode);
  if (rc != CB_OK) return rc;
  alignas(64) CUtensorMap q_map;
  alignas(64) CUtensorMap k_map;
  // dense queries: (d, row, head) with strides (row: 256 B, head: rows_pad*256 B)
  rc = sq::encode_3d(encode, &q_map, dtype, ws + w.qd, head_size, rows_pad, num_kv_heads,
                     head_size * esize, (uint64_t)rows_pad * head_size * esize, sq::kTile, 1);
  if (rc != CB_OK) return rc;
  // keys: (d, kv head, token) with strides (head: 256 B, token: key_token_stride)
  rc = sq::encode_3d(encode, &k_map, dtype, key, head_size, num_kv_heads, num_keys,
                     head_size * esize, key_token_stride, 1, sq::kTile);
  if (rc != CB_OK) return rc;
  if (dtype == CB_DTYPE_BF16) return sq::launch_passes<__nv_bfloat16>(q_map, k_map, c, s);
  return sq::launch_passes<__half>(q_map, k_map, c, s);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory when
// they score: a vLLM worker after the KV cache has claimed the free memory its
// profiler measured (a new allocation there can fail or evict the cache), or a
// host that reaches this library through a C FFI with buffers owned by another
// runtime and no allocator of its own.  cb_sparse_q_scores_static runs the same
// two-pass scorer with its workspace in a file-scope device array instead of a
// caller buffer.  The array (kStaticWorkspaceBytes per GPU) exists on every
// GPU that loads this library, until the process exits.
namespace {
constexpr int64_t kStaticWorkspaceBytes = int64_t(32) << 20;  // 32 MiB
static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

std::mutex g_static_mutex;
// Device address of the array per CUDA context (a device ordinal can name
// several contexts over the process's life: cudaDeviceReset, or an FFI host
// that drives its own context).
cb::ContextTable<void*, 64> g_static_address;

// Device address of the array in the calling thread's current context.  Outside
// a stream capture it is looked up on every call (cudaGetSymbolAddress is a
// table lookup once the module is loaded) and recorded for the context; inside
// a capture only the recorded address is used, so each context needs one call
// outside capture first.
int static_workspace(cudaStream_t stream, void** address) {
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &capture);
  if (e != cudaSuccess) {
    set_error("cb_sparse_q_scores_static: cudaStreamIsCapturing failed: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  void* found = nullptr;
  if (capture == cudaStreamCaptureStatusNone) {
    e = cudaGetSymbolAddress(&found, g_static_workspace);
    if (e != cudaSuccess || found == nullptr) {
      set_error("cb_sparse_q_scores_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return CB_ERR_CUDA;
    }
  }
  void* context = nullptr;
  int rc = current_context(&context);
  if (rc != CB_OK) return rc;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (found != nullptr) {
    if (!g_static_address.store(context, found)) {
      set_error("cb_sparse_q_scores_static: more than 64 CUDA contexts");
      return CB_ERR_INVALID;
    }
  } else {
    found = g_static_address.find(context, nullptr);
    if (found == nullptr) {
      set_error("cb_sparse_q_scores_static: first call in this CUDA context made inside a stream "
                "capture; make one call on each device outside capture first");
      return CB_ERR_INVALID;
    }
  }
  *address = found;
  return CB_OK;
}
}  // namespace

extern "C" int cb_sparse_q_scores_static(const void* query, int64_t query_token_stride,
                                         int64_t num_query_tokens, const void* key,
                                         int64_t key_token_stride, int64_t num_keys,
                                         int64_t num_q_heads, int64_t num_kv_heads,
                                         int64_t head_size, int dtype, const int64_t* query_rows,
                                         const int64_t* query_positions, int64_t num_queries,
                                         float scale, float* scores, int32_t* device_error,
                                         void* stream) {
  CB_BIND(stream, scores);
  int rc = sq::check_shape(num_q_heads, num_kv_heads, head_size, dtype);
  if (rc != CB_OK) return rc;
  rc = sq::check_counts(num_query_tokens, num_keys, num_q_heads, num_kv_heads, num_queries);
  if (rc != CB_OK) return rc;
  int64_t needed = 0;
  rc = cb_sparse_q_workspace_size(num_queries, num_q_heads, num_kv_heads, head_size, dtype, &needed);
  if (rc != CB_OK) return rc;
  // the scorer wants a 1 KiB aligned workspace; the array is 256-B aligned
  constexpr int64_t kUsable = kStaticWorkspaceBytes - 1024;
  CB_REQUIRE(needed <= kUsable,
             "cb_sparse_q_scores_static: %lld queries x %lld/%lld heads need %lld workspace bytes, "
             "above the %lld-byte static workspace; use cb_sparse_q_scores with a caller buffer",
             (long long)num_queries, (long long)num_q_heads, (long long)num_kv_heads,
             (long long)needed, (long long)kUsable);
  void* base = nullptr;
  rc = static_workspace(reinterpret_cast<cudaStream_t>(stream), &base);
  if (rc != CB_OK) return rc;
  const uintptr_t raw = reinterpret_cast<uintptr_t>(base);
  void* aligned = reinterpret_cast<void*>((raw + 1023) & ~static_cast<uintptr_t>(1023));
  return cb_sparse_q_scores(query, query_token_stride, num_query_tokens, key, key_token_stride,
                            num_keys, num_q_heads, num_kv_heads, head_size, dtype, query_rows,
                            query_positions, num_queries, scale, scores, aligned, kUsable,
                            device_error, stream);
}
