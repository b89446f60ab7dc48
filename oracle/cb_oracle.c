/*
 * cb_oracle.c -- CPU restatement of the CacheBlend hot path, used ONLY as
 * test infrastructure: the parity checker of tests/, __graft_entry__.smoke()
 * and the CPU-baseline leg of bench.py.  Nothing in the product links it.
 *
 * Each function restates one piece of the reference (zoudinghong2000/
 * PIC-KVCache, package cacheblend_vllm) in plain C:
 *   orc_paged_gather / orc_paged_scatter  <- kv_layout.py:90-161
 *   orc_relocate                          <- ascend.py:52-103 (cos_sin branch)
 *   orc_blend_load                        <- ascend.py:224-287, 313-370
 *   orc_kv_deviation                      <- ascend.py:535-538
 * Element arithmetic follows torch's per-op semantics for reduced-precision
 * tensors: each op in fp32 (IEEE round-to-nearest; built with
 * -ffp-contract=off), result rounded to nearest-even in the tensor dtype.
 * The deviation sum uses one fixed association order (32 strided lane sums
 * combined by a xor butterfly), the one the CUDA kernel documents, so the two
 * agree bit for bit; any order is a valid restatement of torch.sum.
 * Work is split over OpenMP threads along tokens (nthreads <= 0: all cores).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORC_BF16 = 0, ORC_FP16 = 1, ORC_FP32 = 2 };

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest, ties to even */
  return (uint16_t)(u >> 16);
}

static inline float load_elem(int dtype, const void* p, int64_t i) {
  switch (dtype) {
    case ORC_BF16:
      return bf16_to_f32(((const uint16_t*)p)[i]);
    case ORC_FP16:
      return (float)((const _Float16*)p)[i];
    default:
      return ((const float*)p)[i];
  }
}

static inline void store_elem(int dtype, void* p, int64_t i, float v) {
  switch (dtype) {
    case ORC_BF16:
      ((uint16_t*)p)[i] = f32_to_bf16(v);
      break;
    case ORC_FP16:
      ((_Float16*)p)[i] = (_Float16)v;
      break;
    default:
      ((float*)p)[i] = v;
      break;
  }
}

/* value rounded to the storage dtype and widened back */
static inline float rnd(int dtype, float v) {
  switch (dtype) {
    case ORC_BF16:
      return bf16_to_f32(f32_to_bf16(v));
    case ORC_FP16:
      return (float)(_Float16)v;
    default:
      return v;
  }
}

static inline int64_t wrap_slot(int64_t s, int64_t num_slots) { return s < 0 ? s + num_slots : s; }

int orc_threads(int requested) {
#ifdef _OPENMP
  return requested > 0 ? requested : omp_get_max_threads();
#else
  (void)requested;
  return 1;
#endif
}

/* out[p, t] = plane_p[slot_t // bs, slot_t % bs]; heads of head_bytes each */
int orc_paged_gather(const uint8_t* k, const uint8_t* v, int64_t block_stride, int64_t slot_stride,
                     int64_t head_stride, int64_t num_blocks, int64_t block_size, int64_t heads,
                     int64_t head_bytes, const int64_t* slots, int64_t tokens, uint8_t* out,
                     int64_t out_plane, int64_t out_token, int64_t out_head, int nthreads) {
  const int64_t num_slots = num_blocks * block_size;
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t s = wrap_slot(slots[t], num_slots);
    if (s < 0 || s >= num_slots) return -1;
  }
#pragma omp parallel for schedule(static) num_threads(orc_threads(nthreads))
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t s = wrap_slot(slots[t], num_slots);
    const int64_t blk = s / block_size, off = s % block_size;
    for (int p = 0; p < 2; ++p) {
      const uint8_t* src = (p ? v : k) + blk * block_stride + off * slot_stride;
      uint8_t* dst = out + p * out_plane + t * out_token;
      for (int64_t h = 0; h < heads; ++h) memcpy(dst + h * out_head, src + h * head_stride, head_bytes);
    }
  }
  return 0;
}

/* plane_p[slot_t // bs, slot_t % bs] = src[p, t] (later tokens win on duplicates) */
int orc_paged_scatter(const uint8_t* src, int64_t src_plane, int64_t src_token, int64_t src_head,
                      uint8_t* k, uint8_t* v, int64_t block_stride, int64_t slot_stride,
                      int64_t head_stride, int64_t num_blocks, int64_t block_size, int64_t heads,
                      int64_t head_bytes, const int64_t* slots, int64_t tokens) {
  const int64_t num_slots = num_blocks * block_size;
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t s = wrap_slot(slots[t], num_slots);
    if (s < 0 || s >= num_slots) return -1;
  }
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t s = wrap_slot(slots[t], num_slots);
    const int64_t blk = s / block_size, off = s % block_size;
    for (int p = 0; p < 2; ++p) {
      uint8_t* dst = (p ? v : k) + blk * block_stride + off * slot_stride;
      const uint8_t* from = src + p * src_plane + t * src_token;
      for (int64_t h = 0; h < heads; ++h) memcpy(dst + h * head_stride, from + h * src_head, head_bytes);
    }
  }
  return 0;
}

/*
 * One token row (heads x head_size elements, contiguous) relocated from old
 * to new position.  cos_sin rows hold rotary_dim elements: cos half then sin.
 */
static void relocate_row(int dtype, const void* key, void* out, int64_t row, int64_t heads,
                         int64_t head_size, int64_t rotary_dim, int neox, const void* cos_sin,
                         int64_t old_pos, int64_t new_pos) {
  const int64_t half = rotary_dim / 2;
  const int64_t width = heads * head_size;
  const int64_t oc_base = old_pos * rotary_dim, nc_base = new_pos * rotary_dim;
  for (int64_t i = 0; i < half; ++i) {
    const float oc = load_elem(dtype, cos_sin, oc_base + i);
    const float os = load_elem(dtype, cos_sin, oc_base + half + i);
    const float nc = load_elem(dtype, cos_sin, nc_base + i);
    const float ns = load_elem(dtype, cos_sin, nc_base + half + i);
    /* delta_cos = new_cos*old_cos + new_sin*old_sin; delta_sin = new_sin*old_cos - new_cos*old_sin */
    const float dc = rnd(dtype, rnd(dtype, nc * oc) + rnd(dtype, ns * os));
    const float ds = rnd(dtype, rnd(dtype, ns * oc) - rnd(dtype, nc * os));
    for (int64_t h = 0; h < heads; ++h) {
      const int64_t base = row * width + h * head_size;
      const int64_t ia = neox ? base + i : base + 2 * i;
      const int64_t ib = neox ? base + half + i : base + 2 * i + 1;
      const float a = load_elem(dtype, key, ia);
      const float b = load_elem(dtype, key, ib);
      /* first*dc - second*ds ; second*dc + first*ds */
      store_elem(dtype, out, ia, rnd(dtype, a * dc) - rnd(dtype, b * ds));
      store_elem(dtype, out, ib, rnd(dtype, b * dc) + rnd(dtype, a * ds));
    }
  }
  for (int64_t h = 0; h < heads; ++h) {
    for (int64_t j = rotary_dim; j < head_size; ++j) {
      const int64_t at = row * width + h * head_size + j;
      store_elem(dtype, out, at, load_elem(dtype, key, at));
    }
  }
}

/* key/out: [tokens, heads*head_size] contiguous (out may alias key) */
int orc_relocate(int dtype, const void* key, void* out, int64_t tokens, int64_t heads,
                 int64_t head_size, int64_t rotary_dim, int neox, const void* cos_sin,
                 int64_t max_position, const int64_t* old_pos, const int64_t* new_pos,
                 int nthreads) {
  for (int64_t t = 0; t < tokens; ++t) {
    if (old_pos[t] < 0 || old_pos[t] >= max_position || new_pos[t] < 0 || new_pos[t] >= max_position)
      return -1;
  }
#pragma omp parallel for schedule(static) num_threads(orc_threads(nthreads))
  for (int64_t t = 0; t < tokens; ++t)
    relocate_row(dtype, key, out, t, heads, head_size, rotary_dim, neox, cos_sin, old_pos[t],
                 new_pos[t]);
  return 0;
}

/*
 * One layer of PagedBlendLoader.prefetch into out = contiguous
 * [2, alloc_end, heads*head_size] staging:
 *   1. out[:, :apc] = paged gather of slots[:apc]
 *   2. zero every gap of [apc, alloc_end) not covered by a segment
 *   3. per segment: K relocated (if rotate[s]) and V copied from the host
 *      chunk planes k_src[s] / v_src[s] ([length, heads*head_size] each,
 *      contiguous), placed at rows target[s] .. target[s]+length-1.
 */
int orc_blend_load(int dtype, uint8_t* out, int64_t alloc_end, int64_t apc_prefix,
                   const uint8_t* k_cache, const uint8_t* v_cache, int64_t block_stride,
                   int64_t slot_stride, int64_t head_stride, int64_t num_blocks, int64_t block_size,
                   const int64_t* slots, int64_t heads, int64_t head_size, int64_t rotary_dim,
                   int neox, const void* cos_sin, int64_t max_position, int64_t num_segments,
                   const int64_t* source_start, const int64_t* target_start, const int64_t* length,
                   const int32_t* rotate, const uint64_t* k_src, const uint64_t* v_src,
                   int nthreads) {
  const int64_t esize = dtype == ORC_FP32 ? 4 : 2;
  const int64_t row_bytes = heads * head_size * esize;
  uint8_t* out_k = out;
  uint8_t* out_v = out + alloc_end * row_bytes;
  if (apc_prefix > 0) {
    int rc = orc_paged_gather(k_cache, v_cache, block_stride, slot_stride, head_stride, num_blocks,
                              block_size, heads, head_size * esize, slots, apc_prefix, out,
                              alloc_end * row_bytes, row_bytes, head_size * esize, nthreads);
    if (rc) return rc;
  }
  int64_t cursor = apc_prefix;
  for (int64_t s = 0; s < num_segments; ++s) {
    if (target_start[s] > cursor) {
      memset(out_k + cursor * row_bytes, 0, (target_start[s] - cursor) * row_bytes);
      memset(out_v + cursor * row_bytes, 0, (target_start[s] - cursor) * row_bytes);
    }
    if (target_start[s] + length[s] > cursor) cursor = target_start[s] + length[s];
  }
  if (cursor < alloc_end) {
    memset(out_k + cursor * row_bytes, 0, (alloc_end - cursor) * row_bytes);
    memset(out_v + cursor * row_bytes, 0, (alloc_end - cursor) * row_bytes);
  }
  for (int64_t s = 0; s < num_segments; ++s) {
    if (target_start[s] + length[s] > alloc_end || target_start[s] < apc_prefix) return -1;
    if (rotate[s] && (source_start[s] < 0 || source_start[s] + length[s] > max_position ||
                      target_start[s] + length[s] > max_position))
      return -1;
  }
#pragma omp parallel for schedule(dynamic, 1) num_threads(orc_threads(nthreads))
  for (int64_t s = 0; s < num_segments; ++s) {
    const uint8_t* ks = (const uint8_t*)(uintptr_t)k_src[s];
    const uint8_t* vs = (const uint8_t*)(uintptr_t)v_src[s];
    uint8_t* kd = out_k + target_start[s] * row_bytes;
    memcpy(out_v + target_start[s] * row_bytes, vs, length[s] * row_bytes);
    if (!rotate[s]) {
      memcpy(kd, ks, length[s] * row_bytes);
      continue;
    }
    for (int64_t t = 0; t < length[s]; ++t)
      relocate_row(dtype, ks + t * row_bytes, kd + t * row_bytes, 0, heads, head_size, rotary_dim,
                   neox, cos_sin, source_start[s] + t, target_start[s] + t);
  }
  return 0;
}

/*
 * score[i] = sum_j (fresh[i, j] - cached[abs_i, j])^2 in fp32 with the kernel's
 * association order: the row is cut into units of `unit` elements (16 bytes on
 * the vector path, 1 element otherwise); lane l = q % 32 accumulates unit q's
 * elements in order with fmaf(d, d, acc); the 32 lane sums are combined by a
 * xor butterfly with offsets 16, 8, 4, 2, 1.
 */
int orc_kv_deviation(int dtype, const uint8_t* fresh, int64_t fresh_stride, const uint8_t* cached,
                     int64_t cached_stride, const int64_t* abs_index, int64_t abs_offset,
                     int64_t tokens, int64_t width, int64_t unit, float* scores, int nthreads) {
  if (unit <= 0 || width % unit) return -1;
#pragma omp parallel for schedule(static) num_threads(orc_threads(nthreads))
  for (int64_t i = 0; i < tokens; ++i) {
    const int64_t ai = abs_index ? abs_index[i] : abs_offset + i;
    const uint8_t* f = fresh + i * fresh_stride;
    const uint8_t* c = cached + ai * cached_stride;
    float lane[32];
    for (int l = 0; l < 32; ++l) lane[l] = 0.0f;
    const int64_t units = width / unit;
    for (int64_t q = 0; q < units; ++q) {
      float acc = lane[q % 32];
      for (int64_t e = 0; e < unit; ++e) {
        const float d = load_elem(dtype, f, q * unit + e) - load_elem(dtype, c, q * unit + e);
        acc = fmaf(d, d, acc);
      }
      lane[q % 32] = acc;
    }
    for (int o = 16; o >= 1; o >>= 1) {
      float next[32];
      for (int l = 0; l < 32; ++l) next[l] = lane[l] + lane[l ^ o];
      memcpy(lane, next, sizeof(lane));
    }
    scores[i] = lane[0];
  }
  return 0;
}
