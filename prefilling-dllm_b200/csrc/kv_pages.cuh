// KV page movement: slot-mapped writes into the paged pool (unified and distinct layouts), the reference's
// gather op, and the page<->dense copies used on the prefill/decode boundary.
// All of these are pure byte movement: HBM-bound, 16-byte vectors, one coalesced row segment per thread.
#pragma once

#include "common.cuh"

namespace pdllm {

// ---- unified layout write --------------------------------------------------------------------------
// One thread moves one 16-byte segment of one token's K row and the matching V segment.
// grid.x covers n_tokens * segs_per_row threads; rows are row_bytes long (multiple of 16).
__global__ void store_unified_vec16_kernel(const uint4* __restrict__ key, const uint4* __restrict__ value,
                                           uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                                           const int32_t* __restrict__ slot_mapping, int64_t n_tokens,
                                           int segs_per_row, int64_t key_stride_v, int64_t value_stride_v,
                                           int64_t num_slots, int32_t* status) {
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t total = n_tokens * segs_per_row;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t tok = idx / segs_per_row;
    int seg = static_cast<int>(idx - tok * segs_per_row);
    int64_t slot = slot_mapping[tok];
    if (slot < 0) continue;  // reference: `if slot < 0: return`
    if (slot >= num_slots) {
      if (seg == 0) report_status(status, PDLLM_S_BAD_SLOT);
      continue;
    }
    uint4 kv = key[tok * key_stride_v + seg];
    uint4 vv = value[tok * value_stride_v + seg];
    k_cache[slot * segs_per_row + seg] = kv;
    v_cache[slot * segs_per_row + seg] = vv;
  }
}

// Fallback for rows whose byte length or strides are not multiples of 16: element-size-agnostic bytes.
__global__ void store_unified_bytes_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                                           uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                                           const int32_t* __restrict__ slot_mapping, int64_t n_tokens,
                                           int64_t row_bytes, int64_t key_stride_b, int64_t value_stride_b,
                                           int64_t num_slots, int32_t* status) {
  int64_t tok = blockIdx.x;
  if (tok >= n_tokens) return;
  int64_t slot = slot_mapping[tok];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) report_status(status, PDLLM_S_BAD_SLOT);
    return;
  }
  for (int64_t b = threadIdx.x; b < row_bytes; b += blockDim.x) {
    k_cache[slot * row_bytes + b] = key[tok * key_stride_b + b];
    v_cache[slot * row_bytes + b] = value[tok * value_stride_b + b];
  }
}

// ---- distinct (vLLM) layout write ------------------------------------------------------------------
// K [pages, Hkv, D/x, page_size, x], V [pages, Hkv, D, page_size]. One thread per (token, element).
template <typename E>
__global__ void store_distinct_kernel(const E* __restrict__ key, const E* __restrict__ value,
                                      E* __restrict__ k_cache, E* __restrict__ v_cache,
                                      const int32_t* __restrict__ slot_mapping, int64_t n_tokens,
                                      int num_kv_heads, int head_dim, int page_size, int x,
                                      int64_t key_stride, int64_t value_stride, int64_t num_pages,
                                      int32_t* status) {
  int64_t tok = blockIdx.x;
  if (tok >= n_tokens) return;
  int64_t slot = slot_mapping[tok];
  if (slot < 0) return;
  int64_t page = slot / page_size;
  int off = static_cast<int>(slot - page * page_size);
  if (page >= num_pages) {
    if (threadIdx.x == 0) report_status(status, PDLLM_S_BAD_SLOT);
    return;
  }
  int row = num_kv_heads * head_dim;
  int64_t page_elems = static_cast<int64_t>(row) * page_size;
  for (int e = threadIdx.x; e < row; e += blockDim.x) {
    int h = e / head_dim;
    int d = e - h * head_dim;
    int64_t koff = page * page_elems + (static_cast<int64_t>(h) * (head_dim / x) + d / x) * page_size * x +
                   static_cast<int64_t>(off) * x + (d % x);
    int64_t voff = page * page_elems + (static_cast<int64_t>(h) * head_dim + d) * page_size + off;
    k_cache[koff] = key[tok * key_stride + e];
    v_cache[voff] = value[tok * value_stride + e];
  }
}

// ---- reference gather op (load_kvcache) ---------------------------------------------------------------
// One thread per 16-byte segment of one output row. Output row r of sequence s:
//   r < ctx_len[s]  → cache[block_table[s, r / page_size], r % page_size]
//   else            → new[cu_seqlens_q[s] + r - ctx_len[s]]
__global__ void load_kvcache_kernel(const uint4* __restrict__ k_cache, const uint4* __restrict__ v_cache,
                                    const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
                                    const int32_t* __restrict__ block_table, int64_t bt_stride, int max_pages,
                                    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ cu_k,
                                    const int32_t* __restrict__ ctx_lens, int num_seqs, int segs_per_row,
                                    int page_size, int64_t num_pages, int64_t new_stride_v,
                                    uint4* __restrict__ k_out, uint4* __restrict__ v_out, int64_t total_k,
                                    int32_t* status) {
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t total = total_k * segs_per_row;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t row = idx / segs_per_row;
    int seg = static_cast<int>(idx - row * segs_per_row);
    // binary search the sequence owning this output row
    int lo = 0, hi = num_seqs - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (cu_k[mid] <= row) lo = mid; else hi = mid - 1;
    }
    int s = lo;
    int64_t local = row - cu_k[s];
    int ctx = ctx_lens[s];
    if (local < ctx) {
      int pidx = static_cast<int>(local / page_size);
      int64_t page = (pidx < max_pages) ? block_table[s * bt_stride + pidx] : -1;
      if (page < 0 || page >= num_pages) {
        if (seg == 0) report_status(status, PDLLM_S_BAD_PAGE);
        continue;
      }
      int64_t src = (page * page_size + (local - static_cast<int64_t>(pidx) * page_size)) * segs_per_row + seg;
      k_out[idx] = k_cache[src];
      v_out[idx] = v_cache[src];
    } else {
      int64_t src_row = cu_q[s] + (local - ctx);
      if (src_row >= cu_q[s + 1]) continue;  // row beyond this sequence's new tokens
      k_out[idx] = k_new[src_row * new_stride_v + seg];
      v_out[idx] = v_new[src_row * new_stride_v + seg];
    }
  }
}

// ---- pages <-> dense ---------------------------------------------------------------------------------
template <bool kToPages>
__global__ void page_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                 const int32_t* __restrict__ page_ids, int64_t n_tokens, int page_size,
                                 int segs_per_row, int64_t num_pages, int32_t* status) {
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t total = n_tokens * segs_per_row;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t tok = idx / segs_per_row;
    int seg = static_cast<int>(idx - tok * segs_per_row);
    int64_t page = page_ids[tok / page_size];
    if (page < 0 || page >= num_pages) {
      if (seg == 0) report_status(status, PDLLM_S_BAD_PAGE);
      continue;
    }
    int64_t paged = (page * page_size + tok % page_size) * segs_per_row + seg;
    if (kToPages) dst[paged] = src[idx]; else dst[idx] = src[paged];
  }
}

// ---- pool -> pool ------------------------------------------------------------------------------------
// dst pages := src pages, token by token, for the first n_tokens of the two page lists. The source pool may be another
// GPU's memory mapped through peer access: the loads then cross NVLink directly (plain 16-byte loads, no staging
// buffer, no TMA), which is the prefill -> decode hand-off of the KV of a request.
__global__ void page_to_page_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ src_pages,
                                    uint4* __restrict__ dst, const int32_t* __restrict__ dst_pages, int64_t n_tokens,
                                    int tokens_per_list, int page_size, int segs_per_row, int64_t src_num_pages,
                                    int64_t dst_num_pages, int32_t* status) {
  // the lists hold `tokens_per_list` tokens each (one list per layer and K/V plane, concatenated)
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n_tokens * segs_per_row;
  const int pages_per_list = (tokens_per_list + page_size - 1) / page_size;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = idx / segs_per_row;
    const int seg = static_cast<int>(idx - tok * segs_per_row);
    const int64_t list = tok / tokens_per_list;
    const int64_t t = tok - list * tokens_per_list;
    const int64_t entry = list * pages_per_list + t / page_size;
    const int64_t sp = src_pages[entry], dp = dst_pages[entry];
    if (sp < 0 || sp >= src_num_pages || dp < 0 || dp >= dst_num_pages) {
      if (seg == 0) report_status(status, PDLLM_S_BAD_PAGE);
      continue;
    }
    const int64_t off = t % page_size;
    dst[(dp * page_size + off) * segs_per_row + seg] = src[(sp * page_size + off) * segs_per_row + seg];
  }
}

// ---- per-head compaction -----------------------------------------------------------------------------
// Phase A: staging[j, h, :] = cache[src token keep[h, j], h, :]; phase B: cache[dst token dst_start + j, h, :] =
// staging[j, h, :]. Two launches, so an in-place compaction (dst range overlapping src range) never reads a
// row that was already overwritten. Segments are 16 bytes of one head's D elements.
__global__ void compact_gather_kernel(const uint4* __restrict__ cache, const int32_t* __restrict__ src_pages,
                                      const int64_t* __restrict__ keep, int64_t keep_count, int64_t src_tokens,
                                      int page_size, int num_kv_heads, int segs_per_head, int64_t num_pages,
                                      uint4* __restrict__ staging, int32_t* status) {
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t per_tok = static_cast<int64_t>(num_kv_heads) * segs_per_head;
  int64_t total = keep_count * per_tok;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t j = idx / per_tok;
    int rem = static_cast<int>(idx - j * per_tok);
    int h = rem / segs_per_head;
    int64_t tok = keep[static_cast<int64_t>(h) * keep_count + j];
    if (tok < 0 || tok >= src_tokens) {
      if (rem % segs_per_head == 0) report_status(status, PDLLM_S_BAD_INDEX);
      staging[idx] = make_uint4(0, 0, 0, 0);
      continue;
    }
    int64_t page = src_pages[tok / page_size];
    if (page < 0 || page >= num_pages) {
      if (rem % segs_per_head == 0) report_status(status, PDLLM_S_BAD_PAGE);
      staging[idx] = make_uint4(0, 0, 0, 0);
      continue;
    }
    staging[idx] = cache[(page * page_size + tok % page_size) * per_tok + rem];
  }
}

__global__ void compact_scatter_kernel(uint4* __restrict__ cache, const int32_t* __restrict__ dst_pages,
                                       int64_t keep_count, int64_t dst_start, int page_size, int64_t per_tok,
                                       int64_t num_pages, const uint4* __restrict__ staging, int32_t* status) {
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t total = keep_count * per_tok;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t j = idx / per_tok;
    int64_t rem = idx - j * per_tok;
    int64_t tok = dst_start + j;
    int64_t page = dst_pages[tok / page_size];
    if (page < 0 || page >= num_pages) {
      if (rem == 0) report_status(status, PDLLM_S_BAD_PAGE);
      continue;
    }
    cache[(page * page_size + tok % page_size) * per_tok + rem] = staging[idx];
  }
}

// ---- rotary embedding applied to rows already in pages -----------------------------------------------
// K rows of tokens [start, start + n) were stored UN-rotated; rotate them in place with the table row of each
// token: out = x * cos + rotate_half(x) * sin, every product and the sum rounded to T as the eager model
// computes them (no fused multiply-add). One thread per (token, head, pair i / i + D/2).
template <typename T>
__global__ void rope_pages_kernel(T* __restrict__ cache, const int32_t* __restrict__ page_ids, int64_t start,
                                  int64_t n_tokens, const T* __restrict__ cos_tab, const T* __restrict__ sin_tab,
                                  int page_size, int num_kv_heads, int head_dim, int64_t num_pages,
                                  int32_t* status) {
  const int half = head_dim / 2;
  const int64_t per_tok = static_cast<int64_t>(num_kv_heads) * half;
  const int64_t total = n_tokens * per_tok;
  int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; idx < total; idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t j = idx / per_tok;
    int rem = static_cast<int>(idx - j * per_tok);
    int h = rem / half, i = rem - h * half;
    int64_t tok = start + j;
    int64_t page = page_ids[tok / page_size];
    if (page < 0 || page >= num_pages) {
      if (rem == 0) report_status(status, PDLLM_S_BAD_PAGE);
      continue;
    }
    T* row = cache + ((page * page_size + tok % page_size) * num_kv_heads + h) * head_dim;
    const T* c = cos_tab + j * head_dim;
    const T* s = sin_tab + j * head_dim;
    float x1 = to_f32<T>(row[i]), x2 = to_f32<T>(row[i + half]);
    float a1 = to_f32<T>(from_f32<T>(__fmul_rn(x1, to_f32<T>(c[i]))));
    float b1 = to_f32<T>(from_f32<T>(__fmul_rn(-x2, to_f32<T>(s[i]))));
    float a2 = to_f32<T>(from_f32<T>(__fmul_rn(x2, to_f32<T>(c[i + half]))));
    float b2 = to_f32<T>(from_f32<T>(__fmul_rn(x1, to_f32<T>(s[i + half]))));
    row[i] = from_f32<T>(__fadd_rn(a1, b1));
    row[i + half] = from_f32<T>(__fadd_rn(a2, b2));
  }
}

inline int grid_for(int64_t work_items, int threads) {
  int64_t blocks = (work_items + threads - 1) / threads;
  int64_t cap = static_cast<int64_t>(sm_count()) * 16;  // a few resident CTAs per SM, grid-stride beyond
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace pdllm
