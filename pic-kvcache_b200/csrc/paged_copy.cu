// K1: paged KV gather / scatter between vLLM block-table pages and dense
// [2, T, H, D] tensors (or the chunk-major Store staging).
//
// Semantics follow cacheblend_vllm/kv_layout.py:90-161 (gather_paged_kv /
// scatter_paged_kv): out[plane, t] = cache[plane][slot[t] // bs, slot[t] % bs].
// Design: one warp per (token, plane) row, 16-byte vector moves whenever
// every address and stride allows it, four vectors in flight per lane,
// grid = 8 CTAs x 256 threads per SM with a grid-stride loop.  The op is a
// pure HBM copy (bytes moved = 2 x rows x row_bytes), so the only goals are
// full 512-byte warp transactions and enough bytes in flight per SM.
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

template <bool GATHER>
int launch_paged_copy(PagedDesc pg, DenseDesc dn, const int64_t* slots, int64_t num_tokens,
                      int64_t num_heads, int64_t head_bytes, void* stream, const char* name) {
  // Merge heads into one row when both sides store them back to back.
  if (num_heads > 1 && pg.head_stride == head_bytes && dn.head_stride == head_bytes) {
    head_bytes *= num_heads;
    num_heads = 1;
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
