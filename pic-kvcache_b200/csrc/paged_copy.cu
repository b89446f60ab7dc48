// K1: paged KV gather / scatter between vLLM block-table pages and dense
// [2, T, H, D] tensors (or the chunk-major Store staging).
//
// Semantics follow cacheblend_vllm/kv_layout.py:90-161 (gather_paged_kv /
// scatter_paged_kv): out[plane, t] = cache[plane][slot[t] // bs, slot[t] % bs].
// The op is a pure HBM copy (bytes moved = 2 x rows x row_bytes), so the
// goals are few instructions per byte and enough bytes in flight per SM.
// Two kernels:
//
// * paged_run_kernel (rows contiguous on both sides, vLLM's NHD pages): a
//   vLLM block holds block_size consecutive slots back to back, so the rows
//   of a block-aligned token group usually form one contiguous run on both
//   sides.  One warp per CTA reads a group's slots, checks that they are
//   consecutive inside one block, and lane 0 moves the whole run with one
//   cp.async.bulk load into a shared-memory ring stage and one bulk store
//   out of it (one bulk op per row when the slots are not a run).  The ring
//   is split between loads issued ahead (half the stages) and stores still
//   reading their stage, so both directions keep several runs in flight;
//   waits are bounded and report into a device error word.
// * paged_copy_kernel (any strides, e.g. head-strided HND pages): one warp
//   per (token, plane) row, 16-byte vector moves whenever every address and
//   stride allows it, four vectors in flight per lane, grid = 8 CTAs x 256
//   threads per SM with a grid-stride loop.
#include "cb_async.cuh"
#include "cb_common.cuh"


namespace cb {
namespace {

struct PagedDesc {
  char* k;
  char* v;
  int64_t block_stride;
  int64_t slot_stride;
  int64_t head_stride;
  int64_t num_slots;
  uint32_t block_size;
};

struct DenseDesc {
  char* base;
  int64_t plane_stride;
  int64_t token_stride;
  int64_t head_stride;
  uint32_t chunk_tokens;
  int64_t chunk_stride;
};

__device__ __forceinline__ char* paged_row(const PagedDesc& pg, int plane, int64_t slot) {
  const uint32_t s = static_cast<uint32_t>(slot);
  const uint32_t blk = s / pg.block_size;
  const uint32_t off = s - blk * pg.block_size;
  return (plane ? pg.v : pg.k) + (int64_t)blk * pg.block_stride + (int64_t)off * pg.slot_stride;
}

__device__ __forceinline__ char* dense_row(const DenseDesc& dn, int plane, int64_t t) {
  const uint32_t tt = static_cast<uint32_t>(t);
  const uint32_t c = tt / dn.chunk_tokens;
  const uint32_t r = tt - c * dn.chunk_tokens;
  return dn.base + plane * dn.plane_stride + (int64_t)c * dn.chunk_stride +
         (int64_t)r * dn.token_stride;
}

// Copies one row (num_heads x units_per_head vectors of VB bytes) with the
// whole warp.  Heads are src_hs / dst_hs bytes apart.
template <int VB>
__device__ __forceinline__ void warp_copy_row(const char* src, int64_t src_hs, char* dst,
                                              int64_t dst_hs, uint32_t num_heads,
                                              uint32_t units_per_head, int lane) {
  using V = typename Vec<VB>::T;
  constexpr int U = 4;
  const uint32_t units = num_heads * units_per_head;
  for (uint32_t i0 = lane; i0 < units; i0 += 32 * U) {
    V tmp[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = i0 + u * 32;
      if (i < units) {
        const uint32_t h = i / units_per_head;
        const uint32_t j = i - h * units_per_head;
        tmp[u] = ld_vec(reinterpret_cast<const V*>(src + h * src_hs + (int64_t)j * VB));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t i = i0 + u * 32;
      if (i < units) {
        const uint32_t h = i / units_per_head;
        const uint32_t j = i - h * units_per_head;
        *reinterpret_cast<V*>(dst + h * dst_hs + (int64_t)j * VB) = tmp[u];
      }
    }
  }
}

template <int VB, bool GATHER>
__global__ void __launch_bounds__(256) paged_copy_kernel(PagedDesc pg, DenseDesc dn,
                                                         const int64_t* __restrict__ slots,
                                                         int64_t num_tokens, uint32_t num_heads,
                                                         uint32_t units_per_head) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t tasks = 2 * num_tokens;
  for (int64_t task = warp; task < tasks; task += nwarps) {
    const int64_t t = task >> 1;
    const int plane = static_cast<int>(task & 1);
    int64_t s = __ldg(slots + t);
    if (s < 0) s += pg.num_slots;  // torch advanced-indexing wrap
    if (s < 0 || s >= pg.num_slots) continue;  // rejected by host validation
    char* p = paged_row(pg, plane, s);
    char* d = dense_row(dn, plane, t);
    if (GATHER)
      warp_copy_row<VB>(p, pg.head_stride, d, dn.head_stride, num_heads, units_per_head, lane);
    else
      warp_copy_row<VB>(d, dn.head_stride, p, pg.head_stride, num_heads, units_per_head, lane);
  }
}

// ----------------------------------------------------------- run copy (TMA)
namespace run {
using namespace ::cb::async;

// Run size and CTAs per SM follow the row size (measured on B200, paged
// scatter/gather of 32,768 tokens at block_size 16): one issuing warp per CTA
// keeps only a few runs in flight, so more CTAs per SM win until the ring of
// each gets too shallow.  CB_RUN_UNIT_KB / CB_RUN_CTAS override the policy
// (tuning sweeps only).
#ifndef CB_RUN_UNIT_KB
#define CB_RUN_UNIT_KB 0
#endif
#ifndef CB_RUN_CTAS
#define CB_RUN_CTAS 0
#endif

constexpr uint32_t kMaxStages = 32;
constexpr uint32_t kMaxGroup = 32;  // tokens per unit (one warp reads their slots)
constexpr uint32_t kMinStages = 3;
constexpr size_t kMaxSmem = 227 * 1024;  // opt-in shared memory per CTA
constexpr size_t kSmPool = 228 * 1024;   // shared memory per SM (1 KiB reserved per CTA)

struct Policy {
  uint32_t unit_bytes;  // largest run moved by one bulk load/store pair
  int ctas_per_sm;
};

inline Policy pick_policy(int64_t row_bytes) {
  Policy p{8 * 1024, 4};                                  // rows of 2 KiB and more
  // e.g. one or two 128-dim heads.  5 CTAs per SM, not the 8 that are fastest
  // for a scatter alone (7.1 vs 8.4 us at one head): the loader runs the next
  // layer's load beside each commit on another stream, and with 5 the two
  // kernels share the SMs -- the pipelined load + commit step of a 32,768-token
  // request measured 0.470 vs 0.538 ms at one head and 0.951 vs 1.016 ms at
  // two (B200; 3, 4 and 6 CTAs were slower than 5, and at 1 KiB rows 6 stays).
  if (row_bytes < 1024) p = Policy{4 * 1024, 5};
  else if (row_bytes < 2048) p = Policy{8 * 1024, 6};     // e.g. four heads
  if (CB_RUN_UNIT_KB > 0) p.unit_bytes = CB_RUN_UNIT_KB * 1024;
  if (CB_RUN_CTAS > 0) p.ctas_per_sm = CB_RUN_CTAS;
  return p;
}

struct Geo {
  int64_t num_tokens;
  uint32_t group;        // tokens per unit: a power of two dividing block_size, <= 32
  uint32_t row_bytes;    // one token row of one plane (heads merged), multiple of 16
  uint32_t stages;       // ring depth, >= 3
  uint32_t stage_bytes;  // group * row_bytes rounded up to 128
  uint32_t ring_offset;  // shared-memory offset of the ring
};

struct StageMeta {
  uint32_t rows;        // tokens in the unit
  uint32_t valid;       // bit r: row r has an in-range slot and is copied
  uint32_t src_run;     // source rows are one contiguous run
  uint32_t dst_run;     // destination rows are one contiguous run
  const char* src[kMaxGroup];
  char* dst[kMaxGroup];
};

__device__ int32_t g_error;  // first failure code of any run-copy launch (0: none)

__device__ __forceinline__ void report(int32_t code) { atomicCAS(&g_error, 0, code); }

template <bool GATHER>
__device__ __forceinline__ bool store_unit(uint32_t u, const Geo& geo, uint64_t* bars,
                                           StageMeta* meta, unsigned char* ring, int lane) {
  const uint32_t st = u % geo.stages;
  if (!mbar_wait(&bars[st], (u / geo.stages) & 1u)) return false;
  if (lane == 0) {
    const StageMeta& m = meta[st];
    const unsigned char* buf = ring + static_cast<size_t>(st) * geo.stage_bytes;
    const uint32_t all = m.rows == 32 ? 0xffffffffu : ((1u << m.rows) - 1u);
    fence_async_smem();
    if (m.dst_run && m.valid == all) {
      bulk_store(m.dst[0], buf, m.rows * geo.row_bytes);
    } else {
      for (uint32_t r = 0; r < m.rows; ++r)
        if ((m.valid >> r) & 1u) bulk_store(m.dst[r], buf + r * geo.row_bytes, geo.row_bytes);
    }
    bulk_commit();
  }
  __syncwarp();
  return true;
}

template <bool GATHER>
__global__ void __launch_bounds__(32) paged_run_kernel(PagedDesc pg, DenseDesc dn,
                                                       const int64_t* __restrict__ slots, Geo geo) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  StageMeta* meta = reinterpret_cast<StageMeta*>(smem + kMaxStages * sizeof(uint64_t));
  unsigned char* ring = smem + geo.ring_offset;
  const int lane = threadIdx.x;
  const uint32_t S = geo.stages;
  // loads issued ahead of the oldest pending store (1 <= L <= S - 2)
  const uint32_t L = S - 2;
  // a stage is reloaded S units after its previous load, whose store was
  // issued at unit + L: the S - L - 1 stores issued since may still be reading
  const uint32_t reading = S - L - 1;
  const uint32_t G = geo.group;
  const uint32_t rb = geo.row_bytes;
  if (lane == 0) {
    for (uint32_t i = 0; i < S; ++i) mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncwarp();

  // Group boundaries follow the slots' block alignment: token 0 sits at
  // offset (slot % G) of its group.
  int64_t first = __ldg(slots);
  if (first < 0) first += pg.num_slots;
  const uint32_t phase =
      (first >= 0 && first < pg.num_slots) ? static_cast<uint32_t>(first % G) : 0u;
  const int64_t groups = (geo.num_tokens + phase + G - 1) / G;

  uint32_t it = 0;
  bool ok = true;
  for (int64_t g = blockIdx.x; g < groups && ok; g += gridDim.x) {
    int64_t t0 = g * G - phase;
    int64_t t1 = t0 + G;
    if (t0 < 0) t0 = 0;
    if (t1 > geo.num_tokens) t1 = geo.num_tokens;
    const uint32_t n = static_cast<uint32_t>(t1 - t0);
    int64_t s = -1;
    bool valid = false;
    if (static_cast<uint32_t>(lane) < n) {
      s = __ldg(slots + t0 + lane);
      if (s < 0) s += pg.num_slots;  // torch advanced-indexing wrap
      valid = s >= 0 && s < pg.num_slots;  // out-of-range rows are skipped, as in the row kernel
    }
    const uint32_t all = n == 32 ? 0xffffffffu : ((1u << n) - 1u);
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid) & all;
    const int64_t s0 = __shfl_sync(0xffffffffu, s, 0);
    const int64_t sl = __shfl_sync(0xffffffffu, s, n - 1);
    const bool seq = static_cast<uint32_t>(lane) >= n || s == s0 + lane;
    const bool page_run = __all_sync(0xffffffffu, seq) && vmask == all &&
                          s0 / pg.block_size == sl / pg.block_size;
    const bool dense_run = static_cast<uint32_t>(t0) / dn.chunk_tokens ==
                           static_cast<uint32_t>(t1 - 1) / dn.chunk_tokens;
    int64_t page_off = 0;
    if (valid) {
      const uint32_t blk = static_cast<uint32_t>(s) / pg.block_size;
      const uint32_t off = static_cast<uint32_t>(s) - blk * pg.block_size;
      page_off = static_cast<int64_t>(blk) * pg.block_stride + static_cast<int64_t>(off) * pg.slot_stride;
    }
    for (int plane = 0; plane < 2; ++plane) {
      const uint32_t st = it % S;
      if (lane == 0 && it >= S) bulk_wait_read_dyn(reading);
      __syncwarp();
      StageMeta& m = meta[st];
      if (static_cast<uint32_t>(lane) < n) {
        char* prow = (plane ? pg.v : pg.k) + page_off;
        char* drow = dense_row(dn, plane, t0 + lane);
        m.src[lane] = GATHER ? prow : drow;
        m.dst[lane] = GATHER ? drow : prow;
      }
      if (lane == 0) {
        m.rows = n;
        m.valid = vmask;
        m.src_run = GATHER ? page_run : dense_run;
        m.dst_run = GATHER ? dense_run : page_run;
      }
      __syncwarp();
      if (lane == 0) {
        unsigned char* buf = ring + static_cast<size_t>(st) * geo.stage_bytes;
        mbar_arrive_expect_tx(&bars[st], __popc(vmask) * rb);
        if (m.src_run && vmask == all) {
          bulk_load(buf, m.src[0], n * rb, &bars[st]);
        } else {
          for (uint32_t r = 0; r < n; ++r)
            if ((vmask >> r) & 1u) bulk_load(buf + r * rb, m.src[r], rb, &bars[st]);
        }
      }
      __syncwarp();
      if (it >= L) ok = ok && store_unit<GATHER>(it - L, geo, bars, meta, ring, lane);
      ++it;
    }
  }
  const uint32_t drained = it > L ? it - L : 0;
  for (uint32_t u = drained; u < it; ++u) {
    if (ok) {
      ok = store_unit<GATHER>(u, geo, bars, meta, ring, lane);
    } else {
      // after a failed wait: give the loads still in flight (bounded) time to land
      mbar_wait(&bars[u % S], (u / S) & 1u);
    }
  }
  if (lane == 0) {
    bulk_wait<0>();
    if (!ok) report(1);
  }
}

// Tokens per unit: a power of two <= 32 dividing block_size with a run of at
// most `unit_bytes` (one row when a single row is larger).
uint32_t pick_group(int64_t block_size, int64_t row_bytes, uint32_t unit_bytes) {
  uint32_t g = 1;
  while (g < kMaxGroup && block_size % (2 * g) == 0 && 2 * g * row_bytes <= unit_bytes) g *= 2;
  return g;
}

size_t smem_for(uint32_t stages, uint32_t stage_bytes, uint32_t* ring_offset) {
  size_t off = kMaxStages * sizeof(uint64_t) + stages * sizeof(StageMeta);
  off = (off + 127) / 128 * 128;
  *ring_offset = static_cast<uint32_t>(off);
  return off + static_cast<size_t>(stages) * stage_bytes;
}

// Launches the run kernel when the layout allows it; returns 1 when the
// caller must use the row kernel instead.
template <bool GATHER>
int try_launch(const PagedDesc& pg, const DenseDesc& dn, const int64_t* slots, int64_t num_tokens,
               int64_t num_heads, int64_t row_bytes, cudaStream_t s, const char* name) {
  const uint64_t align = reinterpret_cast<uint64_t>(pg.k) | reinterpret_cast<uint64_t>(pg.v) |
                         reinterpret_cast<uint64_t>(dn.base) | (uint64_t)pg.block_stride |
                         (uint64_t)dn.plane_stride | (uint64_t)dn.chunk_stride | (uint64_t)row_bytes;
  if (num_heads != 1 || (align & 15u) != 0 || pg.slot_stride != row_bytes ||
      dn.token_stride != row_bytes || row_bytes > (int64_t(1) << 20))
    return 1;
  const Policy policy = pick_policy(row_bytes);
  Geo geo{};
  geo.num_tokens = num_tokens;
  geo.group = pick_group(pg.block_size, row_bytes, policy.unit_bytes);
  geo.row_bytes = static_cast<uint32_t>(row_bytes);
  geo.stage_bytes = static_cast<uint32_t>((geo.group * row_bytes + 127) / 128 * 128);
  // fewer CTAs per SM when a CTA's share cannot hold kMinStages stages
  uint32_t ring_offset = 0;
  int ctas = policy.ctas_per_sm;
  auto budget = [](int c) { return c == 1 ? kMaxSmem : kSmPool / c - 1024; };
  while (ctas > 1 && smem_for(kMinStages, geo.stage_bytes, &ring_offset) > budget(ctas)) --ctas;
  uint32_t stages = kMaxStages;
  while (stages >= kMinStages && smem_for(stages, geo.stage_bytes, &ring_offset) > budget(ctas))
    --stages;
  if (stages < kMinStages) return 1;
  geo.stages = stages;
  const size_t smem = smem_for(stages, geo.stage_bytes, &ring_offset);
  geo.ring_offset = ring_offset;
  const int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(paged_run_kernel<GATHER>), smem);
  if (rc != CB_OK) return rc;
  const int64_t groups = (num_tokens + 2 * geo.group - 1) / geo.group;
  const int64_t cap = static_cast<int64_t>(kSmCount) * ctas;
  const int grid = static_cast<int>(groups < cap ? groups : cap);
  paged_run_kernel<GATHER><<<grid, 32, smem, s>>>(pg, dn, slots, geo);
  return launch_status(name);
}

}  // namespace run

template <bool GATHER>
int launch_paged_copy(PagedDesc pg, DenseDesc dn, const int64_t* slots, int64_t num_tokens,
                      int64_t num_heads, int64_t head_bytes, void* stream, const char* name) {
  // Merge heads into one row when both sides store them back to back.
  if (num_heads > 1 && pg.head_stride == head_bytes && dn.head_stride == head_bytes) {
    head_bytes *= num_heads;
    num_heads = 1;
  }
  {
    const int rc = run::try_launch<GATHER>(pg, dn, slots, num_tokens, num_heads, head_bytes,
                                           reinterpret_cast<cudaStream_t>(stream), name);
    if (rc != 1) return rc;
  }
  uint64_t acc = reinterpret_cast<uint64_t>(pg.k) | reinterpret_cast<uint64_t>(pg.v) |
                 (uint64_t)pg.block_stride | (uint64_t)pg.slot_stride |
                 (uint64_t)pg.head_stride | reinterpret_cast<uint64_t>(dn.base) |
                 (uint64_t)dn.plane_stride | (uint64_t)dn.token_stride |
                 (uint64_t)dn.head_stride | (uint64_t)dn.chunk_stride | (uint64_t)head_bytes;
  const int vb = vector_bytes(acc);
  const uint32_t units = static_cast<uint32_t>(head_bytes / vb);
  const int64_t warps_needed = 2 * num_tokens;
  const int64_t blocks_needed = (warps_needed + 7) / 8;
  const int grid = static_cast<int>(blocks_needed < kSmCount * 8 ? blocks_needed : kSmCount * 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint32_t nh = static_cast<uint32_t>(num_heads);
  switch (vb) {
    case 16:
      paged_copy_kernel<16, GATHER><<<grid, 256, 0, s>>>(pg, dn, slots, num_tokens, nh, units);
      break;
    case 8:
      paged_copy_kernel<8, GATHER><<<grid, 256, 0, s>>>(pg, dn, slots, num_tokens, nh, units);
      break;
    case 4:
      paged_copy_kernel<4, GATHER><<<grid, 256, 0, s>>>(pg, dn, slots, num_tokens, nh, units);
      break;
    case 2:
      paged_copy_kernel<2, GATHER><<<grid, 256, 0, s>>>(pg, dn, slots, num_tokens, nh, units);
      break;
    default:
      paged_copy_kernel<1, GATHER><<<grid, 256, 0, s>>>(pg, dn, slots, num_tokens, nh, units);
      break;
  }
  return launch_status(name);
}

int check_common(int64_t num_blocks, int64_t block_size, int64_t num_heads, int64_t head_bytes,
                 int64_t num_tokens, int64_t chunk_tokens) {
  CB_REQUIRE(num_blocks > 0 && block_size > 0, "num_blocks and block_size must be positive");
  CB_REQUIRE(num_blocks * block_size < (int64_t(1) << 31),
             "paged pool of %lld slots exceeds 2^31", (long long)(num_blocks * block_size));
  CB_REQUIRE(num_heads > 0 && head_bytes > 0, "num_heads and head_bytes must be positive");
  CB_REQUIRE(num_heads * head_bytes < (int64_t(1) << 31), "row too large");
  CB_REQUIRE(num_tokens >= 0 && num_tokens < (int64_t(1) << 30), "num_tokens out of range");
  CB_REQUIRE(chunk_tokens < (int64_t(1) << 31), "chunk_tokens out of range");
  return CB_OK;
}

}  // namespace
}  // namespace cb

using namespace cb;

extern "C" int cb_paged_gather(const void* k_cache, const void* v_cache, int64_t block_stride,
                               int64_t slot_stride, int64_t head_stride, int64_t num_blocks,
                               int64_t block_size, int64_t num_heads, int64_t head_bytes,
                               const int64_t* slots, int64_t num_tokens, void* out,
                               int64_t out_plane_stride, int64_t out_token_stride,
                               int64_t out_head_stride, int64_t out_chunk_tokens,
                               int64_t out_chunk_stride, void* stream) {
  CB_BIND(stream, out);
  int rc = check_common(num_blocks, block_size, num_heads, head_bytes, num_tokens,
                        out_chunk_tokens);
  if (rc != CB_OK) return rc;
  if (num_tokens == 0) return CB_OK;
  CB_REQUIRE(k_cache && v_cache && slots && out, "null pointer argument");
  PagedDesc pg{const_cast<char*>(static_cast<const char*>(k_cache)),
               const_cast<char*>(static_cast<const char*>(v_cache)),
               block_stride,
               slot_stride,
               head_stride,
               num_blocks * block_size,
               static_cast<uint32_t>(block_size)};
  DenseDesc dn{static_cast<char*>(out),
               out_plane_stride,
               out_token_stride,
               out_head_stride,
               static_cast<uint32_t>(out_chunk_tokens > 0 ? out_chunk_tokens : (int64_t(1) << 31) - 1),
               out_chunk_tokens > 0 ? out_chunk_stride : 0};
  return launch_paged_copy<true>(pg, dn, slots, num_tokens, num_heads, head_bytes, stream,
                                 "cb_paged_gather");
}

extern "C" int cb_paged_scatter(const void* src, int64_t src_plane_stride,
                                int64_t src_token_stride, int64_t src_head_stride,
                                int64_t src_chunk_tokens, int64_t src_chunk_stride,
                                void* k_cache, void* v_cache, int64_t block_stride,
                                int64_t slot_stride, int64_t head_stride, int64_t num_blocks,
                                int64_t block_size, int64_t num_heads, int64_t head_bytes,
                                const int64_t* slots, int64_t num_tokens, void* stream) {
  CB_BIND(stream, k_cache);
  int rc = check_common(num_blocks, block_size, num_heads, head_bytes, num_tokens,
                        src_chunk_tokens);
  if (rc != CB_OK) return rc;
  if (num_tokens == 0) return CB_OK;
  CB_REQUIRE(k_cache && v_cache && slots && src, "null pointer argument");
  PagedDesc pg{static_cast<char*>(k_cache),
               static_cast<char*>(v_cache),
               block_stride,
               slot_stride,
               head_stride,
               num_blocks * block_size,
               static_cast<uint32_t>(block_size)};
  DenseDesc dn{const_cast<char*>(static_cast<const char*>(src)),
               src_plane_stride,
               src_token_stride,
               src_head_stride,
               static_cast<uint32_t>(src_chunk_tokens > 0 ? src_chunk_tokens : (int64_t(1) << 31) - 1),
               src_chunk_tokens > 0 ? src_chunk_stride : 0};
  return launch_paged_copy<false>(pg, dn, slots, num_tokens, num_heads, head_bytes, stream,
                                  "cb_paged_scatter");
}

extern "C" int cb_paged_copy_error(void* stream, int32_t* value, int reset) {
  CB_BIND(stream, nullptr);
  CB_REQUIRE(value != nullptr, "null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(value, run::g_error, sizeof(int32_t));
  if (e == cudaSuccess && reset) {
    const int32_t zero = 0;
    e = cudaMemcpyToSymbol(run::g_error, &zero, sizeof(int32_t));
  }
  if (e != cudaSuccess) {
    set_error("cb_paged_copy_error: %s", cudaGetErrorString(e));
    return CB_ERR_CUDA;
  }
  return CB_OK;
}
