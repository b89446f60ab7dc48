// Blend attention: the side executor's attention of the computed (possibly
// pruned) queries over the whole staging context, on the 5th-generation
// tensor cores.
//
// Semantics: Qwen3BlendExecutor._attention (cacheblend_vllm/ascend.py:798-846,
// its einsum path).  For query q at absolute position pos_q, query head
// hq = hk * groups + g, and staging key k (position k):
//   w   = round_T(round_T(q . k) * scale)        (bf16/fp16 einsum output, scaled in T)
//   p   = softmax over k <= pos_q of w           (fp32; keys k > pos_q get 0)
//   out = round_T(sum_k p * v)                   (fp32 accumulation)
// The reference rounds the normalized probabilities to T before the second
// product.  Three modes:
//   kNormalized (exact_rounding = 1, the reference's order): two launches over
//     the same tiles.  The first (kRowLse) computes S and each row's
//     log2-sum-exp of w only; the second computes S again and rounds
//     p = 2^(w log2e - lse2) -- the normalized probability -- to T before P V,
//     with no rescaling and no final division.
//   kFlash (exact_rounding = 2): one launch, the unnormalized exp2 values are
//     rounded to T and O is divided by the row sum at the end (flash-attention
//     order), within one T ulp per probability of the reference.
//   kFused (exact_rounding = 0): fp32 logits times the scale, flash order, as
//     the reference's fused NPU kernel computes them.
//
// Layout: rows = (query, group) pairs of one KV head, r = qi * groups + g, in
// 128-row tiles (one 4-D TMA box over the query tensor: 64 dims x groups x 1
// KV head x 128/groups queries, rows in that order), so every K / V
// tile is shared by all groups of the head.  K and V tiles are TMA boxes of the
// staging rows as they lie ([keys][dims], SWIZZLE_128B):
//   S = Q K^T   A = Q tile [rows][dims] (K-major),  B = K tile [keys][dims] (K-major) -> TMEM
//   O += P V    A = P tile [rows][keys] (K-major),  B = V tile [keys][dims] (MN-major) -> TMEM
// An item is (KV head, pair of query tiles = 256 rows); CTAs are persistent and
// take items dealt serpentine, latest queries first.  Per CTA, 12 warps:
//   warp 0   Q loads per item, K tiles through a two-stage ring (TMA)
//   warp 3   V tiles through one slot, loaded once the previous P V has read it
//   warp 1   tcgen05.mma issue: S_A, S_B of key tile t, then P V of tile t-1 for
//            both query tiles, so the tensor core computes ahead of the softmax
//   warp 2   TMEM owner (S_A, S_B, O_A, O_B: 512 columns)
//   warps 4-7 / 8-11  one softmax warpgroup per query tile, a row per thread:
//            read S with tcgen05.ld, apply the reference's roundings and the
//            causal mask, keep an online max / sum in the log2 domain, write P
//            (rounded to T) into shared memory in the SW128 layout the MMA
//            reads, and at the end of an item divide O by the sum and store it.
// While one warpgroup runs its softmax the tensor core works on the other
// tile's products, and each K / V tile serves 256 rows.  O is rescaled
// (tcgen05.ld / st) only when a row's max grows by more than 2^8: until then
// the stale max keeps every exp2 <= 256, and the final division uses the same
// max, so the result is unchanged.
// Every mbarrier wait is bounded (2 s): a wait that runs out records a code in
// *device_error, the CTA drains its MMAs and loads, frees TMEM and returns.
#include <algorithm>
#include <type_traits>

#include "cb_common.cuh"
#include "cb_tcgen05.cuh"

namespace cb {
namespace att {
using namespace ::cb::tc;

constexpr int kHead = 128;
constexpr int kPair = 2;                    // query tiles per item, one softmax warpgroup each
constexpr int kPairRows = kPair * kTile;    // 256 rows per item
constexpr int kKStages = 2;                 // K tiles in flight (V: one, see the producer)
constexpr int kThreads = 384;  // warp 0 Q/K loads, 1 MMA, 2 TMEM owner, 3 V loads; 4-7 / 8-11 softmax
constexpr uint32_t kTmemCols = 512;  // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
constexpr uint32_t kTmemO = 256;
// Register split: 128 control threads x 40 + 256 softmax threads x 232 =
// 64512 = 384 threads x 168, the launch's allocation (__launch_bounds__(384, 1)).
// MMA issue is a few adds per product (split descriptors), so the control roles fit in 40.
constexpr int kRegsControl = 40;
constexpr int kRegsSoftmax = 232;
static_assert(4 * 32 * kRegsControl + 8 * 32 * kRegsSoftmax <= kThreads * 168, "register split");
constexpr float kRescaleLog2 = 8.0f;
constexpr float kLog2e = 1.4426950408889634f;

struct Shared {
  uint64_t q_full, q_empty;
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full, v_empty;
  uint64_t s_full[kPair], s_empty[kPair];
  uint64_t p_full[kPair], pv_done[kPair], o_empty[kPair];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int num_kv_heads;
  int groups;
  int rows_pad;   // multiple of kPairRows
  int q_pairs;    // rows_pad / kPairRows
  int64_t num_queries;
  float scale;
  const int32_t* row_pos;   // [rows_pad]: position of each row, -1 for padding
  const int32_t* pair_max;  // [q_pairs]: largest position among a pair's rows
  float* lse;               // [num_kv_heads][rows_pad]: -(log2-sum-exp of w log2e) per row (kRowLse out, kNormalized in)
  char* out;
  int64_t out_token_stride;  // bytes
  int32_t* error;
};

template <typename T>
__host__ __device__ constexpr uint32_t instr_desc() {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(kTile >> 3) << 17) |
         ((uint32_t)(kTile >> 4) << 24);
}

__device__ __forceinline__ void report(const Params& c, Shared& sh, int code) {
  if (c.error != nullptr) atomicCAS(c.error, 0, code);
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
}
__device__ __forceinline__ bool aborted(Shared& sh) {
  return *reinterpret_cast<volatile int*>(&sh.abort) != 0;
}

__device__ __forceinline__ int cta_item(int k) {
  const int g = static_cast<int>(gridDim.x);
  const int c = static_cast<int>(blockIdx.x);
  return k * g + ((k & 1) ? g - 1 - c : c);
}

// Value rounded to T (round to nearest even) and widened back to fp32.
template <typename T>
__device__ __forceinline__ float round_t(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}
// Two fp32 values rounded to T and packed (low half = a).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// Pairs of fp32 values rounded to T (nearest even) and widened back.  bf16: one
// packed conversion and two bit moves.  Measured against the same rounding done
// on the FMA pipe (Veltkamp splitting): the FMA work slows the tensor core's
// products issued beside it, while the conversion unit still has room next to
// exp2 (1.30 vs 1.48 ms at 32k).
template <typename T>
struct RoundPair;
template <>
struct RoundPair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 apply(float2 y) {
    const uint32_t p = pack2<__nv_bfloat16>(y.x, y.y);
    return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
  }
};
template <>
struct RoundPair<__half> {
  static __device__ __forceinline__ float2 apply(float2 y) {
    return make_float2(round_t<__half>(y.x), round_t<__half>(y.y));
  }
};


__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Modes of attention_kernel.  All but kFused apply the reference einsum path's
// roundings (T logits, T logit * scale); kFused computes fp32 logits times the
// scale, as the reference's fused attention kernel (npu_fused_infer_attention_score,
// ascend.py:814-830) and flash attention do.
constexpr int kFused = 0;
constexpr int kFlash = 1;       // online max / sum, P unnormalized, O divided at the end
constexpr int kRowLse = 2;      // S only: each row's log2-sum-exp into Params::lse
constexpr int kNormalized = 3;  // P = the normalized probabilities from Params::lse

template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap q_map,
                     const __grid_constant__ CUtensorMap k_map,
                     const __grid_constant__ CUtensorMap v_map, Params c) {
  extern __shared__ __align__(1024) unsigned char dyn[];
  __shared__ Shared sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dyn) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* q_buf = base;                                  // kPair Q tiles
  unsigned char* k_buf = base + kPair * kTileBytes;             // kKStages K tiles
  unsigned char* v_buf = k_buf + kKStages * kTileBytes;         // one V tile
  unsigned char* p_buf = v_buf + kTileBytes;                    // kPair P tiles
  const int items = c.num_kv_heads * c.q_pairs;
  constexpr bool EXACT = MODE != kFused;
  constexpr bool LSE_ONLY = MODE == kRowLse;  // no V, no P, no O

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.k_empty[s], 1);
    }
    mbar_init(&sh.v_full, 1);
    mbar_init(&sh.v_empty, 1);
    for (int x = 0; x < kPair; ++x) {
      mbar_init(&sh.s_full[x], 1);
      mbar_init(&sh.s_empty[x], 4);
      mbar_init(&sh.p_full[x], 4);
      mbar_init(&sh.pv_done[x], 1);
      mbar_init(&sh.o_empty[x], 4);
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

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  if (warp == 0) {
    // ------------------------------------------------------ Q and K loads
    if (lane == 0) {
      int t = 0, it = 0;
      uint32_t k_armed = 0, k_parity = 0;  // per stage: a load is in flight / its phase parity
      int q_armed = -1;
      bool ok = true;
      for (int k = 0, item = cta_item(0); item < items && ok && !aborted(sh);
           item = cta_item(++k), ++it) {
        const int qp = c.q_pairs - 1 - item / c.num_kv_heads;
        const int h = item % c.num_kv_heads;
        if (!wait1(&sh.q_empty, (it & 1) ^ 1)) { ok = false; break; }
        mbar_expect_tx(&sh.q_full, kPair * kTileBytes);
        for (int x = 0; x < kPair; ++x) {
          unsigned char* qb = q_buf + x * kTileBytes;
          const int q0 = (qp * kPairRows + x * kTile) / c.groups;  // first query of the tile
          tma_load_4d(qb, &q_map, &sh.q_full, 0, 0, h, q0);
          tma_load_4d(qb + kHalfBytes, &q_map, &sh.q_full, 64, 0, h, q0);
        }
        q_armed = it & 1;
        const int kt_end = max(c.pair_max[qp], 0) / kTile;
        for (int kt = 0; kt <= kt_end; ++kt, ++t) {
          const int s = t % kKStages;
          if (!wait1(&sh.k_empty[s], ((t / kKStages) & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(&sh.k_full[s], kTileBytes);
          unsigned char* kb = k_buf + s * kTileBytes;
          tma_load_3d(kb, &k_map, &sh.k_full[s], 0, h, kt * kTile);
          tma_load_3d(kb + kHalfBytes, &k_map, &sh.k_full[s], 64, h, kt * kTile);
          k_armed |= 1u << s;
          k_parity = (k_parity & ~(1u << s)) | (static_cast<uint32_t>((t / kKStages) & 1) << s);
        }
      }
      if (!ok) report(c, sh, 1);
      // every armed load has landed before the CTA may exit
      for (int s = 0; s < kKStages; ++s)
        if ((k_armed >> s) & 1u) wait1(&sh.k_full[s], (k_parity >> s) & 1u);
      if (q_armed >= 0) wait1(&sh.q_full, q_armed);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------ V loads
    // V(t) may land only after P V of tile t-1 has read the previous one;
    // it is needed after S(t+1), so its latency hides behind those products.
    if (lane == 0 && !LSE_ONLY) {
      int t = 0;
      int v_armed = -1;
      bool ok = true;
      for (int k = 0, item = cta_item(0); item < items && ok && !aborted(sh); item = cta_item(++k)) {
        const int qp = c.q_pairs - 1 - item / c.num_kv_heads;
        const int h = item % c.num_kv_heads;
        const int kt_end = max(c.pair_max[qp], 0) / kTile;
        for (int kt = 0; kt <= kt_end; ++kt, ++t) {
          if (!wait1(&sh.v_empty, (t & 1) ^ 1)) { ok = false; break; }
          mbar_expect_tx(&sh.v_full, kTileBytes);
          tma_load_3d(v_buf, &v_map, &sh.v_full, 0, h, kt * kTile);
          tma_load_3d(v_buf + kHalfBytes, &v_map, &sh.v_full, 64, h, kt * kTile);
          v_armed = t & 1;
        }
      }
      if (!ok) report(c, sh, 1);
      if (v_armed >= 0) wait1(&sh.v_full, v_armed);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = instr_desc<T>();
      const uint32_t idesc_bmn = idesc | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(q_buf);
      const uint32_t k_addr = smem_u32(k_buf);
      const uint32_t v_addr = smem_u32(v_buf);
      const uint32_t p_addr = smem_u32(p_buf);
      int t = 0, it = 0;
      bool ok = true;
      // O_x += P_x V for tile u of the current item, both query tiles
      auto issue_pv = [&](int u, bool first_of_item) -> bool {
        if (!wait1(&sh.v_full, u & 1)) return false;
        for (int x = 0; x < kPair; ++x) {
          if (!wait1(&sh.p_full[x], u & 1)) return false;
          if (first_of_item && !wait1(&sh.o_empty[x], (it & 1) ^ 1)) return false;
          tc_fence_after();
          umma_k128_bmn(sh.tmem_base + kTmemO + x * kTile, p_addr + x * kTileBytes, v_addr,
                        idesc_bmn, !first_of_item);
          umma_commit(&sh.pv_done[x]);
        }
        umma_commit(&sh.v_empty);
        return true;
      };
      for (int k = 0, item = cta_item(0); item < items && ok && !aborted(sh);
           item = cta_item(++k), ++it) {
        const int qp = c.q_pairs - 1 - item / c.num_kv_heads;
        if (!wait1(&sh.q_full, it & 1)) { ok = false; break; }
        const int kt_end = max(c.pair_max[qp], 0) / kTile;
        for (int kt = 0; kt <= kt_end; ++kt, ++t) {
          const int s = t % kKStages;
          if (!wait1(&sh.k_full[s], (t / kKStages) & 1)) { ok = false; break; }
          const uint32_t kb = k_addr + s * kTileBytes;
          for (int x = 0; x < kPair; ++x) {
            if (!wait1(&sh.s_empty[x], (t & 1) ^ 1)) { ok = false; break; }
            tc_fence_after();
            umma_k128(sh.tmem_base + x * kTile, q_addr + x * kTileBytes, kb, idesc, false);
            umma_commit(&sh.s_full[x]);
          }
          if (!ok) break;
          umma_commit(&sh.k_empty[s]);
          if (!LSE_ONLY && kt > 0 && !issue_pv(t - 1, kt == 1)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        umma_commit(&sh.q_empty);  // every S of this item issued: Q may be replaced
        if (!LSE_ONLY && !issue_pv(t - 1, kt_end == 0)) {
          ok = false;
          break;
        }
      }
      if (!ok) report(c, sh, 2);
      umma_commit(&sh.drain);
      wait1(&sh.drain, 0);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // ------------------------------------------------------ softmax / epilogue
    const int x = (warp - 4) >> 2;           // query tile of the pair
    const int ew = warp & 3;                 // TMEM lanes 32*ew .. +31
    const int row_in_tile = ew * 32 + lane;  // this thread's row
    const uint32_t lane_off = static_cast<uint32_t>(ew * 32) << 16;
    const uint32_t s_tmem = sh.tmem_base + x * kTile + lane_off;
    const uint32_t o_tmem = sh.tmem_base + kTmemO + x * kTile + lane_off;
    unsigned char* my_p = p_buf + x * kTileBytes;
    int t = 0;
    bool ok = true;
    for (int k = 0, item = cta_item(0); item < items && ok; item = cta_item(++k)) {
      const int qp = c.q_pairs - 1 - item / c.num_kv_heads;
      const int h = item % c.num_kv_heads;
      const int r = qp * kPairRows + x * kTile + row_in_tile;
      const int pos = c.row_pos[r];
      const int kt_end = max(c.pair_max[qp], 0) / kTile;
      float m_used = -INFINITY;  // log2-domain max the exponentials are taken against
      float l = 0.0f;
      // kNormalized: -(log2-sum-exp) of the row, so p = 2^(w log2e + neg_lse) is normalized
      const float neg_lse = MODE == kNormalized ? c.lse[static_cast<int64_t>(h) * c.rows_pad + r] : 0.0f;
      for (int kt = 0; kt <= kt_end; ++kt, ++t) {
        if (!wait_warp(&sh.s_full[x], t & 1)) { ok = false; break; }
        tc_fence_after();
        uint32_t v[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(s_tmem + q * 32, v[q]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.s_empty[x]);
        // EXACT: the reference's roundings, w = T(T(s) * scale); fused: w = s (the
        // scale is folded into the exp2 argument below); keys > pos masked
        const int valid = min(max(pos - kt * kTile + 1, 0), kTile);
        float2 w[64];
        const float2 sc2 = make_float2(c.scale, c.scale);
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float2 sv = make_float2(__uint_as_float(v[j >> 4][(2 * j) & 31]),
                                        __uint_as_float(v[j >> 4][(2 * j + 1) & 31]));
          if constexpr (EXACT)
            w[j] = RoundPair<T>::apply(__fmul2_rn(RoundPair<T>::apply(sv), sc2));
          else
            w[j] = sv;
        }
        if (valid < kTile) {  // this row's position ends inside the tile
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            if (2 * j >= valid) w[j].x = -INFINITY;
            if (2 * j + 1 >= valid) w[j].y = -INFINITY;
          }
        }
        // log2-domain multiplier: log2e, or scale * log2e when the scale is folded in
        const float mul = EXACT ? kLog2e : c.scale * kLog2e;
        float2 nm;  // the exponent offset of this tile's p
        if constexpr (MODE == kNormalized) {
          nm = make_float2(neg_lse, neg_lse);
        } else {
          float mx[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) mx[i] = -INFINITY;
#pragma unroll
          for (int j = 0; j < 64; ++j) mx[j & 3] = max3(mx[j & 3], w[j].x, w[j].y);
          // w times a positive multiplier, and rounding is monotonic, so
          // max(w) * mul = max(w * mul)
          const float tile_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * mul;
          const bool grow =
              tile_max > m_used + kRescaleLog2 || (m_used == -INFINITY && tile_max > -INFINITY);
          // the P buffer is free and O settled once the previous tile's P V is done
          if (!LSE_ONLY && kt > 0 && !wait_warp(&sh.pv_done[x], (t - 1) & 1)) { ok = false; break; }
          if (__any_sync(0xffffffffu, grow)) {
            const float m_new = grow ? tile_max : m_used;
            const float corr = grow ? (m_used == -INFINITY ? 0.0f : ex2(m_used - m_new)) : 1.0f;
            if (!LSE_ONLY && kt > 0) {  // O holds earlier tiles of this item: rescale its rows
              tc_fence_after();
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint32_t o[32];
                tmem_ld32(o_tmem + q * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * corr);
                tmem_st32(o_tmem + q * 32, o);
              }
              tmem_wait_st();
            }
            l *= corr;
            m_used = m_new;
          }
          // a padding row keeps m_used = -inf: its p are exact zeros
          const float base_m = m_used == -INFINITY ? 0.0f : m_used;
          nm = make_float2(-base_m, -base_m);
        }
        if (MODE == kNormalized && kt > 0 && !wait_warp(&sh.pv_done[x], (t - 1) & 1)) { ok = false; break; }
        // p = 2^(w mul + offset): rounded to T into the SW128 P tile (not in kRowLse);
        // the sum in fp32 (not in kNormalized)
        const float2 l2e = make_float2(mul, mul);
        float2 sm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sm[i] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16) {  // 16-byte chunk of 8 keys
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 xe = __ffma2_rn(w[c16 * 4 + e], l2e, nm);
            const float2 pe = make_float2(ex2(xe.x), ex2(xe.y));
            if constexpr (MODE != kNormalized) sm[e] = __fadd2_rn(sm[e], pe);
            if constexpr (!LSE_ONLY) packed[e] = pack2<T>(pe.x, pe.y);
          }
          if constexpr (!LSE_ONLY) {
            const int half = c16 >> 3;
            const int chunk = c16 & 7;
            unsigned char* dst = my_p + half * kHalfBytes + row_in_tile * 128 +
                                 ((chunk ^ (row_in_tile & 7)) * 16);
            *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          }
        }
        if constexpr (MODE != kNormalized) {
          const float2 s01 = __fadd2_rn(sm[0], sm[1]);
          const float2 s23 = __fadd2_rn(sm[2], sm[3]);
          const float2 st = __fadd2_rn(s01, s23);
          l += st.x + st.y;
        }
        if constexpr (!LSE_ONLY) {
          fence_async_smem();  // generic-proxy P writes -> the MMA's async-proxy reads
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sh.p_full[x]);
        }
      }
      if (!ok) break;
      if constexpr (LSE_ONLY) {
        // -(m + log2 l); a padding row (no key) stores 0 and is never read
        c.lse[static_cast<int64_t>(h) * c.rows_pad + r] = l > 0.0f ? -(m_used + lg2(l)) : 0.0f;
        continue;
      }
      // O of this item complete once the last P V is done
      if (!wait_warp(&sh.pv_done[x], (t - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const int64_t qi = static_cast<int64_t>(r) / c.groups;
      const int g = r - static_cast<int>(qi) * c.groups;
      const bool store = qi < c.num_queries && pos >= 0;
      // kNormalized: P was normalized, O is the output; else divide by the row sum
      const float inv = !store ? 0.0f : (MODE == kNormalized ? 1.0f : (l > 0.0f ? 1.0f / l : 0.0f));
      T* dst = reinterpret_cast<T*>(c.out + qi * c.out_token_stride) +
               static_cast<int64_t>(h * c.groups + g) * kHead;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t o[32];
        tmem_ld32(o_tmem + q * 32, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const uint4 wv = make_uint4(pack2<T>(__uint_as_float(o[j]) * inv, __uint_as_float(o[j + 1]) * inv),
                                        pack2<T>(__uint_as_float(o[j + 2]) * inv, __uint_as_float(o[j + 3]) * inv),
                                        pack2<T>(__uint_as_float(o[j + 4]) * inv, __uint_as_float(o[j + 5]) * inv),
                                        pack2<T>(__uint_as_float(o[j + 6]) * inv, __uint_as_float(o[j + 7]) * inv));
            *reinterpret_cast<uint4*>(dst + q * 32 + j) = wv;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.o_empty[x]);
    }
    if (!ok && lane == 0) report(c, sh, 3);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(sh.tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// Row positions (rows past the last query: -1) and the largest position of
// each pair of query tiles.  A position past the last key sees every key, as
// the reference's mask (q_pos < k_pos over the staging rows) lets it: it is
// clamped to num_keys - 1.
__device__ __forceinline__ int32_t clamp_position(int64_t pos, int64_t num_keys) {
  return static_cast<int32_t>(pos < num_keys ? (pos < -1 ? -1 : pos) : num_keys - 1);
}
__global__ void __launch_bounds__(256) prep_kernel(const int64_t* __restrict__ positions,
                                                   int64_t num_queries, int64_t num_keys, int groups,
                                                   int rows_pad, int32_t* __restrict__ row_pos,
                                                   int32_t* __restrict__ pair_max) {
  const int lane = threadIdx.x & 31;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t threads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = tid; r < rows_pad; r += threads) {
    const int64_t qi = r / groups;
    row_pos[r] = qi < num_queries ? clamp_position(positions[qi], num_keys) : -1;
  }
  const int q_pairs = rows_pad / kPairRows;
  for (int64_t qt = tid >> 5; qt < q_pairs; qt += threads >> 5) {
    int mx = -1;
    for (int r = lane; r < kPairRows; r += 32) {
      const int64_t qi = (qt * kPairRows + r) / groups;
      if (qi < num_queries) mx = max(mx, static_cast<int>(clamp_position(positions[qi], num_keys)));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) pair_max[qt] = mx;
  }
}

// ---------------------------------------------------------------- host side
struct Workspace {
  size_t row_pos, pair_max, lse, total;
  int64_t rows_pad;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Workspace layout(int64_t num_queries, int64_t num_keys, int64_t num_q_heads, int64_t num_kv_heads) {
  const int64_t groups = num_q_heads / num_kv_heads;
  Workspace w{};
  w.rows_pad = (num_queries * groups + kPairRows - 1) / kPairRows * kPairRows;
  size_t off = 0;
  w.row_pos = off;
  off = align_up(off + (size_t)w.rows_pad * 4, 256);
  w.pair_max = off;
  off = align_up(off + (size_t)(w.rows_pad / kPairRows) * 4, 256);
  w.lse = off;  // the normalized mode's row log2-sum-exps
  off = align_up(off + (size_t)num_kv_heads * w.rows_pad * 4, 256);
  w.total = off;
  return w;
}

// kPair Q tiles, kKStages K tiles, one V tile, kPair P tiles (+ 1 KiB alignment slack)
constexpr size_t kDynSmem = 1024 + (2 * kPair + kKStages + 1) * kTileBytes;
static_assert(kDynSmem + 1024 <= 232448, "shared memory per CTA (static part padded to 1 KiB)");

int check_shape(int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size, int dtype) {
  CB_SUPPORTED(dtype == CB_DTYPE_BF16 || dtype == CB_DTYPE_FP16,
               "blend attention needs bf16 or fp16 query / key / value");
  CB_SUPPORTED(head_size == kHead, "blend attention supports head_size 128 (got %lld)",
               (long long)head_size);
  CB_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
             "query heads must be a multiple of KV heads");
  const int64_t groups = num_q_heads / num_kv_heads;
  CB_SUPPORTED(groups <= kTile && kTile % groups == 0, "query groups must divide 128");
  return CB_OK;
}

}  // namespace att
}  // namespace cb

using namespace cb;

extern "C" int cb_blend_attention_workspace_size(int64_t num_queries, int64_t num_keys,
                                                 int64_t num_q_heads, int64_t num_kv_heads,
                                                 int64_t head_size, int dtype, int64_t* bytes) {
  clear_error();
  CB_REQUIRE(bytes != nullptr, "null output");
  int rc = att::check_shape(num_q_heads, num_kv_heads, head_size, dtype);
  if (rc != CB_OK) return rc;
  CB_REQUIRE(num_queries >= 0 && num_keys >= 0, "negative size");
  *bytes = static_cast<int64_t>(att::layout(num_queries, num_keys, num_q_heads, num_kv_heads).total);
  return CB_OK;
}

extern "C" int cb_blend_attention(const void* query, int64_t query_token_stride, const void* key,
                                  int64_t key_token_stride, const void* value,
                                  int64_t value_token_stride, int64_t num_keys, int64_t num_q_heads,
                                  int64_t num_kv_heads, int64_t head_size, int dtype,
                                  const int64_t* query_positions, int64_t num_queries, float scale,
                                  int exact_rounding, void* out, int64_t out_token_stride,
                                  void* workspace, int64_t workspace_bytes, int32_t* device_error,
                                  void* stream) {
  CB_BIND(stream, out);
  int rc = att::check_shape(num_q_heads, num_kv_heads, head_size, dtype);
  if (rc != CB_OK) return rc;
  CB_REQUIRE(num_queries >= 0 && num_keys >= 0, "negative size");
  if (num_queries == 0) return CB_OK;
  CB_REQUIRE(num_keys > 0, "attention needs at least one key");
  CB_REQUIRE(query && key && value && query_positions && out && workspace, "null pointer argument");
  CB_REQUIRE(num_keys < (int64_t(1) << 31) && num_queries * (num_q_heads / num_kv_heads) < (int64_t(1) << 30),
             "size out of range");
  const uint64_t acc = reinterpret_cast<uint64_t>(query) | reinterpret_cast<uint64_t>(key) |
                       reinterpret_cast<uint64_t>(value) | reinterpret_cast<uint64_t>(out) |
                       (uint64_t)query_token_stride | (uint64_t)key_token_stride |
                       (uint64_t)value_token_stride | (uint64_t)out_token_stride |
                       reinterpret_cast<uint64_t>(workspace);
  CB_SUPPORTED((acc & 15u) == 0, "blend attention needs 16-byte aligned rows and strides");
  const att::Workspace w = att::layout(num_queries, num_keys, num_q_heads, num_kv_heads);
  CB_REQUIRE(workspace_bytes >= static_cast<int64_t>(w.total), "workspace too small (%lld < %zu)",
             (long long)workspace_bytes, w.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int groups = static_cast<int>(num_q_heads / num_kv_heads);
  {
    const int64_t blocks = std::max<int64_t>((w.rows_pad + 255) / 256, w.rows_pad / att::kPairRows / 8 + 1);
    const int grid = static_cast<int>(std::min<int64_t>(blocks, kSmCount * 4));
    att::prep_kernel<<<grid, 256, 0, s>>>(query_positions, num_queries, num_keys, groups,
                                           static_cast<int>(w.rows_pad),
                                           reinterpret_cast<int32_t*>(ws + w.row_pos),
                                           reinterpret_cast<int32_t*>(ws + w.pair_max));
    rc = launch_status("cb_blend_attention (prep)");
    if (rc != CB_OK) return rc;
  }
  tc::EncodeTiled encode = nullptr;
  rc = tc::get_encoder(&encode);
  if (rc != CB_OK) return rc;
  CUtensorMap q_map, k_map, v_map;
  {
    // query [num_queries][num_kv_heads * groups][128] as (dims, group, KV head, query)
    const uint64_t dims[4] = {static_cast<uint64_t>(head_size), static_cast<uint64_t>(groups),
                              static_cast<uint64_t>(num_kv_heads), static_cast<uint64_t>(num_queries)};
    const uint64_t strides[3] = {static_cast<uint64_t>(head_size * 2),
                                 static_cast<uint64_t>(groups * head_size * 2),
                                 static_cast<uint64_t>(query_token_stride)};
    rc = tc::encode_4d(encode, &q_map, dtype, query, dims, strides, static_cast<uint32_t>(groups), 1,
                       static_cast<uint32_t>(tc::kTile / groups));
  }
  if (rc == CB_OK)
    rc = tc::encode_3d(encode, &k_map, dtype, key, head_size, num_kv_heads, num_keys, head_size * 2,
                       key_token_stride, 1, tc::kTile);
  if (rc == CB_OK)
    rc = tc::encode_3d(encode, &v_map, dtype, value, head_size, num_kv_heads, num_keys,
                       head_size * 2, value_token_stride, 1, tc::kTile);
  if (rc != CB_OK) return rc;
  att::Params c{};
  c.num_kv_heads = static_cast<int>(num_kv_heads);
  c.groups = groups;
  c.rows_pad = static_cast<int>(w.rows_pad);
  c.q_pairs = static_cast<int>(w.rows_pad / att::kPairRows);
  c.num_queries = num_queries;
  c.scale = scale;
  c.row_pos = reinterpret_cast<const int32_t*>(ws + w.row_pos);
  c.pair_max = reinterpret_cast<const int32_t*>(ws + w.pair_max);
  c.lse = reinterpret_cast<float*>(ws + w.lse);
  c.out = static_cast<char*>(out);
  c.out_token_stride = out_token_stride;
  c.error = device_error;
  const int grid = static_cast<int>(std::min<int64_t>(num_kv_heads * c.q_pairs, kSmCount));
  CB_REQUIRE(exact_rounding >= 0 && exact_rounding <= 2, "exact_rounding must be 0, 1 or 2 (got %d)",
             exact_rounding);
  CB_REQUIRE(exact_rounding || scale > 0.0f,
             "the fused-logit mode needs a positive scale (got %g)", static_cast<double>(scale));
  const bool bf16 = dtype == CB_DTYPE_BF16;
  // exact_rounding 1: the row log2-sum-exps, then the products with normalized P
  const int modes[2] = {exact_rounding == 1 ? att::kRowLse : (exact_rounding == 2 ? att::kFlash : att::kFused),
                        exact_rounding == 1 ? att::kNormalized : -1};
  for (int mode : modes) {
    if (mode < 0) break;
    void (*kernel)(CUtensorMap, CUtensorMap, CUtensorMap, att::Params) = nullptr;
    switch (mode) {
      case att::kFused:
        kernel = bf16 ? att::attention_kernel<__nv_bfloat16, att::kFused> : att::attention_kernel<__half, att::kFused>;
        break;
      case att::kFlash:
        kernel = bf16 ? att::attention_kernel<__nv_bfloat16, att::kFlash> : att::attention_kernel<__half, att::kFlash>;
        break;
      case att::kRowLse:
        kernel = bf16 ? att::attention_kernel<__nv_bfloat16, att::kRowLse> : att::attention_kernel<__half, att::kRowLse>;
        break;
      default:
        kernel = bf16 ? att::attention_kernel<__nv_bfloat16, att::kNormalized>
                      : att::attention_kernel<__half, att::kNormalized>;
        break;
    }
    rc = ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), att::kDynSmem);
    if (rc != CB_OK) return rc;
    kernel<<<grid, att::kThreads, att::kDynSmem, s>>>(q_map, k_map, v_map, c);
    rc = launch_status("cb_blend_attention");
    if (rc != CB_OK) return rc;
  }
  return CB_OK;
}
