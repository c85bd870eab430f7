// extern "C" surface of libpdllm_b200.so: argument validation and kernel launches.
// Declarations and the reference op each entry replaces: include/pdllm_b200.h.
#include "attn_simt.cuh"
#include "attn_decode_sm100.cuh"
#include "attn_sm100.cuh"
#include "common.cuh"
#include "dense.cuh"
#include "gemm_sm100.cuh"
#include "kv_pages.cuh"
#include "score.cuh"

#include <cstdlib>
#include <mutex>

using namespace pdllm;

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename F>
int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case PDLLM_F32: return f(static_cast<float*>(nullptr));
    case PDLLM_BF16: return f(static_cast<__nv_bfloat16*>(nullptr));
    case PDLLM_F16: return f(static_cast<__half*>(nullptr));
    default: return fail(PDLLM_E_INVALID, "unknown dtype %d", dtype);
  }
}

}  // namespace

extern "C" {

int pdllm_abi_version(void) { return PDLLM_ABI_VERSION; }

const char* pdllm_last_error(void) { return last_error_ref().c_str(); }

int pdllm_device_supported(void) {
  int dev = 0, major = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return fail(-static_cast<int>(e), "no usable CUDA device: %s", cudaGetErrorString(e));
  return major == 10 ? 1 : 0;
}

// ------------------------------------------------------------------------------------------------ (5)
int pdllm_store_kvcache_unified(const void* key, const void* value, void* k_cache, void* v_cache,
                                const int32_t* slot_mapping, int64_t n_tokens, int64_t row_elems,
                                int64_t key_stride, int64_t value_stride, int elem_bytes,
                                int64_t num_slots, int32_t* status, void* stream) {
  if (n_tokens < 0 || row_elems <= 0 || num_slots < 0 || elem_bytes <= 0)
    return fail(PDLLM_E_INVALID, "store_kvcache_unified: bad sizes (n_tokens=%lld row_elems=%lld)", (long long)n_tokens, (long long)row_elems);
  if (n_tokens == 0) return 0;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return fail(PDLLM_E_INVALID, "store_kvcache_unified: null pointer");
  const int64_t row_bytes = row_elems * elem_bytes;
  const bool vec = (row_bytes % 16 == 0) && ((key_stride * elem_bytes) % 16 == 0) && ((value_stride * elem_bytes) % 16 == 0) &&
                   aligned16(key) && aligned16(value) && aligned16(k_cache) && aligned16(v_cache);
  if (vec) {
    const int segs = static_cast<int>(row_bytes / 16);
    const int threads = 256;
    (void)launch_dependent(store_unified_vec16_kernel, dim3(grid_for(n_tokens * segs, threads)), dim3(threads), 0, as_stream(stream),
        static_cast<const uint4*>(key), static_cast<const uint4*>(value), static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache),
        slot_mapping, n_tokens, segs, key_stride * elem_bytes / 16, value_stride * elem_bytes / 16, num_slots, status);
  } else {
    store_unified_bytes_kernel<<<static_cast<unsigned>(n_tokens), 128, 0, as_stream(stream)>>>(
        static_cast<const uint8_t*>(key), static_cast<const uint8_t*>(value), static_cast<uint8_t*>(k_cache),
        static_cast<uint8_t*>(v_cache), slot_mapping, n_tokens, row_bytes, key_stride * elem_bytes, value_stride * elem_bytes,
        num_slots, status);
  }
  return check_launch("store_kvcache_unified");
}

int pdllm_store_kvcache_distinct(const void* key, const void* value, void* k_cache, void* v_cache,
                                 const int32_t* slot_mapping, int64_t n_tokens, int num_kv_heads,
                                 int head_dim, int page_size, int x, int64_t key_stride,
                                 int64_t value_stride, int elem_bytes, int64_t num_pages,
                                 int32_t* status, void* stream) {
  if (n_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || x <= 0 || head_dim % x != 0)
    return fail(PDLLM_E_INVALID, "store_kvcache_distinct: bad shape (Hkv=%d D=%d page=%d x=%d)", num_kv_heads, head_dim, page_size, x);
  if (n_tokens == 0) return 0;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return fail(PDLLM_E_INVALID, "store_kvcache_distinct: null pointer");
  const unsigned grid = static_cast<unsigned>(n_tokens);
  if (elem_bytes == 2) {
    store_distinct_kernel<uint16_t><<<grid, 128, 0, as_stream(stream)>>>(
        static_cast<const uint16_t*>(key), static_cast<const uint16_t*>(value), static_cast<uint16_t*>(k_cache),
        static_cast<uint16_t*>(v_cache), slot_mapping, n_tokens, num_kv_heads, head_dim, page_size, x, key_stride, value_stride,
        num_pages, status);
  } else if (elem_bytes == 4) {
    store_distinct_kernel<uint32_t><<<grid, 128, 0, as_stream(stream)>>>(
        static_cast<const uint32_t*>(key), static_cast<const uint32_t*>(value), static_cast<uint32_t*>(k_cache),
        static_cast<uint32_t*>(v_cache), slot_mapping, n_tokens, num_kv_heads, head_dim, page_size, x, key_stride, value_stride,
        num_pages, status);
  } else if (elem_bytes == 1) {
    store_distinct_kernel<uint8_t><<<grid, 128, 0, as_stream(stream)>>>(
        static_cast<const uint8_t*>(key), static_cast<const uint8_t*>(value), static_cast<uint8_t*>(k_cache),
        static_cast<uint8_t*>(v_cache), slot_mapping, n_tokens, num_kv_heads, head_dim, page_size, x, key_stride, value_stride,
        num_pages, status);
  } else {
    return fail(PDLLM_E_INVALID, "store_kvcache_distinct: elem_bytes %d not in {1,2,4}", elem_bytes);
  }
  return check_launch("store_kvcache_distinct");
}

int pdllm_load_kvcache(const void* k_cache, const void* v_cache, const void* k_new, const void* v_new,
                       const int32_t* block_table, int64_t block_table_stride, int max_pages,
                       const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                       const int32_t* context_lens, int num_seqs, int num_kv_heads, int head_dim,
                       int page_size, int64_t num_pages, int64_t new_stride, int elem_bytes,
                       void* k_out, void* v_out, int64_t total_k, int32_t* status, void* stream) {
  if (num_seqs <= 0 || total_k < 0 || page_size <= 0) return fail(PDLLM_E_INVALID, "load_kvcache: bad sizes");
  if (total_k == 0) return 0;
  if (!k_new || !v_new || !cu_seqlens_q || !cu_seqlens_k || !context_lens || !k_out || !v_out)
    return fail(PDLLM_E_INVALID, "load_kvcache: null pointer");
  // the caches and the block table are read only for sequences with a cached context: without pages there is none
  if ((num_pages > 0 || max_pages > 0) && (!k_cache || !v_cache || !block_table))
    return fail(PDLLM_E_INVALID, "load_kvcache: null cache or block_table with num_pages=%lld max_pages=%d", (long long)num_pages, max_pages);
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * elem_bytes;
  if (row_bytes % 16 != 0 || (new_stride * elem_bytes) % 16 != 0 || !aligned16(k_cache) || !aligned16(v_cache) ||
      !aligned16(k_new) || !aligned16(v_new) || !aligned16(k_out) || !aligned16(v_out))
    return fail(PDLLM_E_UNSUPPORTED, "load_kvcache: rows must be 16-byte multiples and 16-byte aligned");
  const int segs = static_cast<int>(row_bytes / 16);
  load_kvcache_kernel<<<grid_for(total_k * segs, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(k_cache), static_cast<const uint4*>(v_cache), static_cast<const uint4*>(k_new),
      static_cast<const uint4*>(v_new), block_table, block_table_stride, max_pages, cu_seqlens_q, cu_seqlens_k, context_lens,
      num_seqs, segs, page_size, num_pages, new_stride * elem_bytes / 16, static_cast<uint4*>(k_out), static_cast<uint4*>(v_out),
      total_k, status);
  return check_launch("load_kvcache");
}

// ------------------------------------------------------------------------------------------------ (3)+(1)
static int validate_attn(const pdllm_attn_params* p) {
  if (p == nullptr) return fail(PDLLM_E_INVALID, "paged_attention: null params");
  if (p->total_q < 0 || p->num_seqs < 0) return fail(PDLLM_E_INVALID, "paged_attention: negative sizes");
  if (p->total_q == 0 || p->num_seqs == 0) return 0;
  if (!p->q || !p->k_new || !p->v_new || !p->out || !p->cu_seqlens_q) return fail(PDLLM_E_INVALID, "paged_attention: null tensor pointer");
  if (p->num_q_heads <= 0 || p->num_kv_heads <= 0 || p->head_dim <= 0 || p->num_q_heads % p->num_kv_heads != 0)
    return fail(PDLLM_E_INVALID, "paged_attention: bad head configuration Hq=%d Hkv=%d D=%d", p->num_q_heads, p->num_kv_heads, p->head_dim);
  if (p->kv_layout != PDLLM_KV_NONE) {
    if (!p->k_cache || !p->v_cache || !p->block_table || !p->seq_lens || p->page_size <= 0)
      return fail(PDLLM_E_INVALID, "paged_attention: cache layout %d needs cache, block_table, seq_lens and page_size", p->kv_layout);
    if (p->kv_layout == PDLLM_KV_DISTINCT && (p->x <= 0 || p->head_dim % p->x != 0))
      return fail(PDLLM_E_INVALID, "paged_attention: distinct layout needs x dividing head_dim");
  }
  if (!(p->sm_scale > 0.f)) return fail(PDLLM_E_INVALID, "paged_attention: sm_scale must be positive");
  if (p->mask_mode != PDLLM_MASK_BLOCK && p->mask_mode != PDLLM_MASK_CAUSAL) return fail(PDLLM_E_INVALID, "paged_attention: unknown mask_mode %d", p->mask_mode);
  if (p->max_query_len <= 0) return fail(PDLLM_E_INVALID, "paged_attention: max_query_len must be positive");
  return 1;
}

int pdllm_attn_select_impl(const pdllm_attn_params* p) {
  int v = validate_attn(p);
  if (v < 0) return v;
  if (p->impl == PDLLM_ATTN_SIMT) return PDLLM_ATTN_SIMT;
  const char* why = nullptr;
  const bool ok = tc::supported(p, &why);
  if (p->impl == PDLLM_ATTN_TC) return ok ? PDLLM_ATTN_TC : fail(PDLLM_E_UNSUPPORTED, "tcgen05 attention: %s", why);
  return ok ? PDLLM_ATTN_TC : PDLLM_ATTN_SIMT;
}

int pdllm_attn_uses_cluster_kernel(const pdllm_attn_params* p) {
  const int impl = pdllm_attn_select_impl(p);
  if (impl < 0) return impl;
  return (impl == PDLLM_ATTN_TC && dec::make_plan(p).use && !getenv("PDLLM_NO_DECODE_KERNEL")) ? 1 : 0;
}

int64_t pdllm_attn_workspace_bytes(const pdllm_attn_params* p) {
  int impl = pdllm_attn_select_impl(p);
  if (impl < 0) return impl;
  if (impl != PDLLM_ATTN_TC) return 0;
  if (!getenv("PDLLM_NO_DECODE_KERNEL")) {
    const dec::Plan dp = dec::make_plan(p);
    if (dp.use) {     // enough for either form, should no cluster size fit on the device
      const int64_t a = dec::workspace_bytes(dp), b = tc::workspace_bytes(p);
      return a > b ? a : b;
    }
  }
  return tc::workspace_bytes(p);
}

int pdllm_paged_attention(const pdllm_attn_params* p, void* stream) {
  int v = validate_attn(p);
  if (v <= 0) return v;
  int impl = pdllm_attn_select_impl(p);
  if (impl < 0) return impl;
  if (impl == PDLLM_ATTN_TC) {
    // few (sequence, KV head, query tile) units: one query tile per CTA, splits merged inside a thread-block cluster
    const dec::Plan dp = dec::make_plan(p);
    if (dp.use && p->total_q > 0 && !getenv("PDLLM_NO_DECODE_KERNEL")) {
      const int rc = dec::launch(p, dp, as_stream(stream));
      if (rc != PDLLM_E_UNSUPPORTED) return rc;      // else: no cluster size fits on this device
    }
    return tc::launch(p, as_stream(stream));
  }
  return launch_attn_simt(p, as_stream(stream));
}

// ------------------------------------------------------------------------------------------------ (4)
int64_t pdllm_unmask_workspace_bytes(int block_len) {
  if (block_len <= 0) return 0;
  return unmask_ws_words(block_len) * 4;
}

int pdllm_unmask_step(const void* logits, int64_t logits_stride, const void* last_logit, int dtype,
                      int block_len, int64_t vocab, int shift, int64_t* block_ids, int64_t mask_id,
                      float threshold, int conf_dtype, int32_t* out_counts, float* out_conf,
                      int64_t* out_x0, void* workspace, int64_t workspace_bytes, void* stream) {
  return pdllm_unmask_step_batched(logits, logits_stride, 0, last_logit, 0, dtype, 1, block_len, vocab, shift, block_ids, mask_id,
                                   threshold, conf_dtype, out_counts, out_conf, out_x0, workspace, workspace_bytes, stream);
}

int pdllm_unmask_step_batched(const void* logits, int64_t logits_stride, int64_t batch_stride, const void* last_logit,
                              int64_t last_stride, int dtype, int batch, int block_len, int64_t vocab, int shift,
                              int64_t* block_ids, int64_t mask_id, float threshold, int conf_dtype, int32_t* out_counts,
                              float* out_conf, int64_t* out_x0, void* workspace, int64_t workspace_bytes, void* stream) {
  if (batch < 0 || batch > 65535) return fail(PDLLM_E_INVALID, "unmask_step: batch %d must be in [0, 65535]", batch);
  if (batch == 0) return 0;
  if (block_len <= 0 || block_len > kUnmaskMaxBlock || vocab <= 0 || vocab >= (1ll << 31))
    return fail(PDLLM_E_INVALID, "unmask_step: block_len %d must be in [1,%d], vocab %lld in [1, 2^31)", block_len, kUnmaskMaxBlock, (long long)vocab);
  if (!logits || !block_ids) return fail(PDLLM_E_INVALID, "unmask_step: null pointer");
  if (conf_dtype != PDLLM_F32 && conf_dtype != PDLLM_BF16 && conf_dtype != PDLLM_F16) return fail(PDLLM_E_INVALID, "unmask_step: bad conf_dtype %d", conf_dtype);
  if (!workspace || workspace_bytes < batch * pdllm_unmask_workspace_bytes(block_len))
    return fail(PDLLM_E_WORKSPACE, "unmask_step: workspace of %lld bytes required", (long long)(batch * pdllm_unmask_workspace_bytes(block_len)));
  dim3 grid(kUnmaskChunks, block_len, batch);
  return dispatch_dtype(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    (void)launch_dependent(unmask_kernel<T>, grid, dim3(kUnmaskThreads), 0, as_stream(stream),
        static_cast<const T*>(logits), logits_stride, static_cast<const T*>(last_logit), block_len, vocab, shift, block_ids, mask_id,
        threshold, conf_dtype, out_counts, out_conf, out_x0, static_cast<float*>(workspace), batch_stride, last_stride);
    return check_launch("unmask_kernel");
  });
}

// Scratch of pdllm_unmask_step_static: lives in the library image, one copy per GPU that loads the library, held
// until the process exits. Sized for PDLLM_UNMASK_STATIC_MAX_BLOCK slots (about 7 KB).
static __device__ __align__(256) float g_unmask_static_scratch[(PDLLM_UNMASK_STATIC_MAX_BLOCK * (3 * kUnmaskChunks + 3) + 1 + 63) / 64 * 64];

// The array's name is only a host-side handle: the device address has to be looked up, per device, with that device
// current. Done on the first call for a device and cached.
// `refresh` drops the cached address first: a cudaDeviceReset (or any re-creation of the device's primary context)
// invalidates it, which shows up as an invalid-value error from the next use.
static int unmask_static_scratch_ptr(float** out, bool refresh = false) {
  static std::mutex mu;
  static float* cached[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(PDLLM_E_UNSUPPORTED, "unmask_step_static: device ordinal %d not supported", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (refresh) cached[dev] = nullptr;
  if (cached[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_unmask_static_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(e != cudaSuccess ? static_cast<int>(e) : PDLLM_E_DRIVER, "cudaGetSymbolAddress(unmask scratch): %s", cudaGetErrorString(e));
    cached[dev] = static_cast<float*>(ptr);
  }
  *out = cached[dev];
  return 0;
}

int pdllm_unmask_step_static(const void* logits, int64_t logits_stride, const void* last_logit, int dtype,
                             int block_len, int64_t vocab, int shift, int64_t* block_ids, int64_t mask_id,
                             float threshold, int conf_dtype, int32_t* out_counts, float* out_conf,
                             int64_t* out_x0, void* stream) {
  if (block_len > PDLLM_UNMASK_STATIC_MAX_BLOCK)
    return fail(PDLLM_E_INVALID, "unmask_step_static: block_len %d exceeds the built-in scratch (max %d); use pdllm_unmask_step with a caller workspace",
                block_len, PDLLM_UNMASK_STATIC_MAX_BLOCK);
  if (block_len <= 0) return fail(PDLLM_E_INVALID, "unmask_step_static: block_len must be positive");
  float* scratch = nullptr;
  int rc = unmask_static_scratch_ptr(&scratch);
  if (rc != 0) return rc;
  // The counters at the tail of the scratch must be zero when the kernel starts. The kernel leaves them zeroed, but
  // the array is shared by every call and keeps whatever an interrupted call left: clear them on the stream first.
  const int64_t words = unmask_ws_words(block_len);
  const int64_t counter_words = block_len + 1;
  cudaError_t e = cudaMemsetAsync(scratch + (words - counter_words), 0, counter_words * 4, as_stream(stream));
  if (e == cudaErrorInvalidValue || e == cudaErrorInvalidDevicePointer || e == cudaErrorContextIsDestroyed) {
    // the address cached for this device went stale (its context was reset since): look it up again, once
    (void)cudaGetLastError();
    if ((rc = unmask_static_scratch_ptr(&scratch, true)) != 0) return rc;
    e = cudaMemsetAsync(scratch + (words - counter_words), 0, counter_words * 4, as_stream(stream));
  }
  if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return pdllm_unmask_step(logits, logits_stride, last_logit, dtype, block_len, vocab, shift, block_ids, mask_id, threshold,
                           conf_dtype, out_counts, out_conf, out_x0, scratch, words * 4, stream);
}

// ------------------------------------------------------------------------------------------------ (2a)(2b)
int pdllm_self_information_scores(const void* rows, int64_t row_stride, int dtype, int n_chunks,
                                  int n_labels, int64_t vocab, const int64_t* labels,
                                  float* scores_out, float* nll_out, int32_t* status, void* stream) {
  if (n_chunks < 0 || n_labels < 0 || vocab <= 0) return fail(PDLLM_E_INVALID, "self_information_scores: bad sizes");
  if (n_chunks == 0) return 0;
  if (!scores_out) return fail(PDLLM_E_INVALID, "self_information_scores: null scores_out");
  if (n_labels > 0 && (!rows || !labels || !nll_out))
    return fail(PDLLM_E_INVALID, "self_information_scores: rows, labels and nll_out are required when n_labels > 0");
  if (n_labels > 0) {
    int rc = dispatch_dtype(dtype, [&](auto* tag) -> int {
      using T = std::remove_pointer_t<decltype(tag)>;
      self_info_nll_kernel<T><<<static_cast<unsigned>(n_chunks) * n_labels, kScoreThreads, 0, as_stream(stream)>>>(
          static_cast<const T*>(rows), row_stride, n_labels, vocab, labels, nll_out, status);
      return check_launch("self_info_nll_kernel");
    });
    if (rc != 0) return rc;
  }
  self_info_mean_kernel<<<(n_chunks + 127) / 128, 128, 0, as_stream(stream)>>>(nll_out, n_chunks, n_labels, scores_out);
  return check_launch("self_info_mean_kernel");
}

int pdllm_topk_chunks(const float* scores, int n_chunks, int topk, int keep_first,
                      int32_t* selected_out, int32_t* count_out, void* stream) {
  if (n_chunks < 0 || n_chunks > 1024) return fail(PDLLM_E_INVALID, "topk_chunks: n_chunks %d must be in [0,1024]", n_chunks);
  if (!count_out) return fail(PDLLM_E_INVALID, "topk_chunks: null count_out");
  if (n_chunks > 0 && (!scores || !selected_out)) return fail(PDLLM_E_INVALID, "topk_chunks: null pointer");
  int threads = ((n_chunks > 0 ? n_chunks : 1) + 31) / 32 * 32;
  topk_chunks_kernel<<<1, threads, 0, as_stream(stream)>>>(scores, n_chunks, topk, keep_first, selected_out, count_out);
  return check_launch("topk_chunks_kernel");
}

// ------------------------------------------------------------------------------------------------ (2c)
int64_t pdllm_evict_workspace_bytes(int num_q_heads, int query_len, int64_t key_len) {
  if (num_q_heads <= 0 || query_len <= 0 || key_len <= 0) return 0;
  return static_cast<int64_t>(num_q_heads) * query_len * key_len * 4;
}

int pdllm_query_to_chunk_scores(const void* q, const void* k, int dtype, int64_t key_len,
                                int num_q_heads, int num_kv_heads, int head_dim, int prefix_len,
                                int chunk_len, int query_len, float scale, int reduce_mean, int causal,
                                float* out, void* workspace, int64_t workspace_bytes, void* stream) {
  if (chunk_len <= 0 || query_len <= 0) return 0;  // the reference returns an empty tensor
  if (!q || !k || !out) return fail(PDLLM_E_INVALID, "query_to_chunk_scores: null pointer");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return fail(PDLLM_E_INVALID, "query_to_chunk_scores: num_query_heads must be divisible by num_kv_heads");
  if (head_dim <= 0 || head_dim > 256) return fail(PDLLM_E_INVALID, "query_to_chunk_scores: unsupported head_dim %d", head_dim);
  if (query_len > 64) return fail(PDLLM_E_INVALID, "query_to_chunk_scores: query_len=%d is too large (max 64)", query_len);
  if (static_cast<int64_t>(prefix_len) + chunk_len + query_len > key_len)
    return fail(PDLLM_E_INVALID, "query_to_chunk_scores: prefix+chunk+query exceeds the sequence length");
  const int64_t need = pdllm_evict_workspace_bytes(num_q_heads, query_len, key_len);
  if (!workspace || workspace_bytes < need) return fail(PDLLM_E_WORKSPACE, "query_to_chunk_scores: workspace of %lld bytes required", (long long)need);
  const int query_start = prefix_len + chunk_len;
  const size_t smem_a = (static_cast<size_t>(kEvictKeys) * (head_dim + 1) + static_cast<size_t>(query_len) * head_dim) * 4;
  dim3 grid_a(static_cast<unsigned>((key_len + kEvictKeys - 1) / kEvictKeys), num_q_heads);
  int rc = dispatch_dtype(dtype, [&](auto* tag) -> int {
    using T = std::remove_pointer_t<decltype(tag)>;
    if (smem_a > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(evict_logits_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_a));
      if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    evict_logits_kernel<T><<<grid_a, kEvictThreads, smem_a, as_stream(stream)>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), key_len, num_q_heads, num_kv_heads, head_dim, query_start, query_len,
        scale, causal, static_cast<float*>(workspace));
    return check_launch("evict_logits_kernel");
  });
  if (rc != 0) return rc;
  evict_reduce_kernel<<<num_q_heads, kEvictThreads, 2 * query_len * sizeof(float), as_stream(stream)>>>(
      static_cast<const float*>(workspace), key_len, query_len, prefix_len, chunk_len, reduce_mean, out);
  return check_launch("evict_reduce_kernel");
}

int pdllm_evict_select(const float* head_scores, int n_layers, int num_q_heads, int num_kv_heads,
                       int chunk_len, int pool_kernel, int granularity, int keep_count, int force_first,
                       int largest, int64_t* keep_out, float* pooled_out, void* stream) {
  if (!head_scores || !keep_out) return fail(PDLLM_E_INVALID, "evict_select: null pointer");
  if (n_layers <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || chunk_len <= 0)
    return fail(PDLLM_E_INVALID, "evict_select: bad shape");
  if (keep_count <= 0 || keep_count > chunk_len) return fail(PDLLM_E_INVALID, "evict_select: keep_count %d must be in [1, chunk_len=%d]", keep_count, chunk_len);
  if (granularity != 0 && granularity != 1) return fail(PDLLM_E_INVALID, "evict_select: granularity must be 0 (global) or 1 (per_head)");
  const int rows = granularity == 0 ? 1 : n_layers * num_kv_heads;
  const size_t smem = static_cast<size_t>(chunk_len) * 8;
  if (smem > 200 * 1024) return fail(PDLLM_E_UNSUPPORTED, "evict_select: chunk_len %d too large", chunk_len);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(evict_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  evict_select_kernel<<<rows, kSelectThreads, smem, as_stream(stream)>>>(head_scores, n_layers, num_q_heads, num_kv_heads, chunk_len,
                                                                        pool_kernel, granularity, keep_count, force_first, largest,
                                                                        keep_out, pooled_out);
  return check_launch("evict_select_kernel");
}

// ------------------------------------------------------------------------------------------------ PD boundary
int pdllm_gather_pages(const void* cache, const int32_t* page_ids, int64_t n_tokens, int page_size,
                       int64_t row_elems, int elem_bytes, int64_t num_pages, void* out,
                       int32_t* status, void* stream) {
  if (n_tokens < 0 || page_size <= 0 || row_elems <= 0) return fail(PDLLM_E_INVALID, "gather_pages: bad sizes");
  if (n_tokens == 0) return 0;
  if (!cache || !page_ids || !out) return fail(PDLLM_E_INVALID, "gather_pages: null pointer");
  const int64_t row_bytes = row_elems * elem_bytes;
  if (row_bytes % 16 != 0 || !aligned16(cache) || !aligned16(out)) return fail(PDLLM_E_UNSUPPORTED, "gather_pages: rows must be 16-byte multiples");
  const int segs = static_cast<int>(row_bytes / 16);
  page_copy_kernel<false><<<grid_for(n_tokens * segs, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(cache), static_cast<uint4*>(out), page_ids, n_tokens, page_size, segs, num_pages, status);
  return check_launch("gather_pages");
}

int pdllm_scatter_pages(const void* src, const int32_t* page_ids, int64_t n_tokens, int page_size,
                        int64_t row_elems, int elem_bytes, int64_t num_pages, void* cache,
                        int32_t* status, void* stream) {
  if (n_tokens < 0 || page_size <= 0 || row_elems <= 0) return fail(PDLLM_E_INVALID, "scatter_pages: bad sizes");
  if (n_tokens == 0) return 0;
  if (!cache || !page_ids || !src) return fail(PDLLM_E_INVALID, "scatter_pages: null pointer");
  const int64_t row_bytes = row_elems * elem_bytes;
  if (row_bytes % 16 != 0 || !aligned16(cache) || !aligned16(src)) return fail(PDLLM_E_UNSUPPORTED, "scatter_pages: rows must be 16-byte multiples");
  const int segs = static_cast<int>(row_bytes / 16);
  page_copy_kernel<true><<<grid_for(n_tokens * segs, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(cache), page_ids, n_tokens, page_size, segs, num_pages, status);
  return check_launch("scatter_pages");
}

// ------------------------------------------------------------------------------------------------ dense row ops
#define PDLLM_DISPATCH_DTYPE(dtype, what, ...)                                    \
  do {                                                                            \
    if ((dtype) == PDLLM_F32) { using T = float; __VA_ARGS__; }                   \
    else if ((dtype) == PDLLM_BF16) { using T = __nv_bfloat16; __VA_ARGS__; }     \
    else if ((dtype) == PDLLM_F16) { using T = __half; __VA_ARGS__; }             \
    else return fail(PDLLM_E_UNSUPPORTED, what ": dtype must be f32, bf16 or f16"); \
  } while (0)

int pdllm_add_rmsnorm(void* x, const void* delta, const void* weight, void* out, int64_t n_tokens, int hidden, int64_t x_stride,
                      int64_t delta_stride, int64_t out_stride, float eps, int dtype, void* stream) {
  if (n_tokens < 0 || hidden <= 0) return fail(PDLLM_E_INVALID, "add_rmsnorm: bad sizes");
  if (n_tokens == 0) return 0;
  if (!x || !weight || !out) return fail(PDLLM_E_INVALID, "add_rmsnorm: null pointer");
  if (dtype != PDLLM_F32 && hidden % 8 == 0 && hidden <= 8 * 1024 && x_stride % 8 == 0 && out_stride % 8 == 0 &&
      (delta == nullptr || (delta_stride % 8 == 0 && aligned16(delta))) && aligned16(x) && aligned16(weight) && aligned16(out)) {
    const int vec_threads = ((hidden / 8 + 31) / 32) * 32;          // one 16-byte vector per thread
    if (dtype == PDLLM_BF16)
      (void)launch_dependent(add_rmsnorm_vec_kernel<__nv_bfloat16>, dim3(static_cast<unsigned>(n_tokens)), dim3(vec_threads), 0, as_stream(stream),
                             static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(delta), static_cast<const __nv_bfloat16*>(weight),
                             static_cast<__nv_bfloat16*>(out), hidden, x_stride, delta_stride, out_stride, eps);
    else
      (void)launch_dependent(add_rmsnorm_vec_kernel<__half>, dim3(static_cast<unsigned>(n_tokens)), dim3(vec_threads), 0, as_stream(stream),
                             static_cast<__half*>(x), static_cast<const __half*>(delta), static_cast<const __half*>(weight),
                             static_cast<__half*>(out), hidden, x_stride, delta_stride, out_stride, eps);
    return check_launch("add_rmsnorm");
  }
  const int threads = hidden >= 2048 ? 512 : 256;
  PDLLM_DISPATCH_DTYPE(dtype, "add_rmsnorm",
                       (void)launch_dependent(add_rmsnorm_kernel<T>, dim3(static_cast<unsigned>(n_tokens)), dim3(threads), 0, as_stream(stream),
                           static_cast<T*>(x), static_cast<const T*>(delta), static_cast<const T*>(weight), static_cast<T*>(out), hidden,
                           x_stride, delta_stride, out_stride, eps));
  return check_launch("add_rmsnorm");
}

int pdllm_rope_inplace(void* x, const void* cos_tab, const void* sin_tab, int64_t n_tokens, int num_heads, int head_dim,
                       int64_t row_stride, int dtype, void* stream) {
  if (n_tokens < 0 || num_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0) return fail(PDLLM_E_INVALID, "rope_inplace: bad sizes");
  if (n_tokens == 0) return 0;
  if (!x || !cos_tab || !sin_tab) return fail(PDLLM_E_INVALID, "rope_inplace: null pointer");
  const int grid = grid_for(n_tokens * num_heads * (head_dim / 2), 256);
  PDLLM_DISPATCH_DTYPE(dtype, "rope_inplace",
                       (void)launch_dependent(rope_inplace_kernel<T>, dim3(grid), dim3(256), 0, as_stream(stream), static_cast<T*>(x), static_cast<const T*>(cos_tab),
                                                                                   static_cast<const T*>(sin_tab), n_tokens, num_heads,
                                                                                   head_dim, row_stride));
  return check_launch("rope_inplace");
}

int pdllm_rope_store(void* qkv, int64_t row_stride, const void* cos_tab, const void* sin_tab, int64_t n_tokens, int num_q_heads,
                     int num_kv_heads, int head_dim, void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t num_slots,
                     int k_before_rotation, int dtype, int32_t* status, void* stream) {
  if (n_tokens < 0 || num_q_heads < 0 || num_kv_heads < 0 || num_q_heads + num_kv_heads <= 0 || head_dim <= 0)
    return fail(PDLLM_E_INVALID, "rope_store: bad sizes");
  if (n_tokens == 0) return 0;
  if (!qkv || !cos_tab || !sin_tab) return fail(PDLLM_E_INVALID, "rope_store: null pointer");
  if (slot_mapping != nullptr && (!k_cache || !v_cache || num_slots <= 0)) return fail(PDLLM_E_INVALID, "rope_store: slot mapping without caches");
  if (dtype != PDLLM_BF16 && dtype != PDLLM_F16) return fail(PDLLM_E_UNSUPPORTED, "rope_store: 16-bit dtypes only (use rope_inplace + store_kvcache_unified)");
  if (head_dim % 16 != 0 || row_stride % 8 != 0 || row_stride < static_cast<int64_t>(num_q_heads + 2 * num_kv_heads) * head_dim ||
      !aligned16(qkv) || !aligned16(cos_tab) || !aligned16(sin_tab) || (slot_mapping != nullptr && (!aligned16(k_cache) || !aligned16(v_cache))))
    return fail(PDLLM_E_UNSUPPORTED, "rope_store: head_dim must be a multiple of 16 and every row 16-byte aligned");
  const int64_t work = n_tokens * (num_q_heads + 2 * num_kv_heads) * (head_dim / 16);
  const int grid = grid_for(work, 128);
  if (dtype == PDLLM_BF16)
    (void)launch_dependent(rope_store_kernel<__nv_bfloat16>, dim3(grid), dim3(128), 0, as_stream(stream), static_cast<__nv_bfloat16*>(qkv),
                           static_cast<const __nv_bfloat16*>(cos_tab), static_cast<const __nv_bfloat16*>(sin_tab), n_tokens, num_q_heads, num_kv_heads,
                           head_dim, row_stride, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), slot_mapping, num_slots,
                           k_before_rotation, status);
  else
    (void)launch_dependent(rope_store_kernel<__half>, dim3(grid), dim3(128), 0, as_stream(stream), static_cast<__half*>(qkv),
                           static_cast<const __half*>(cos_tab), static_cast<const __half*>(sin_tab), n_tokens, num_q_heads, num_kv_heads, head_dim,
                           row_stride, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), slot_mapping, num_slots, k_before_rotation, status);
  return check_launch("rope_store");
}

int pdllm_silu_mul(const void* gate_up, void* out, int64_t n_tokens, int inter, int64_t gu_stride, int64_t out_stride, int dtype,
                   void* stream) {
  if (n_tokens < 0 || inter <= 0) return fail(PDLLM_E_INVALID, "silu_mul: bad sizes");
  if (n_tokens == 0) return 0;
  if (!gate_up || !out) return fail(PDLLM_E_INVALID, "silu_mul: null pointer");
  const int grid = grid_for(n_tokens * inter, 256);
  PDLLM_DISPATCH_DTYPE(dtype, "silu_mul",
                       silu_mul_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<const T*>(gate_up), static_cast<T*>(out), n_tokens,
                                                                               inter, gu_stride, out_stride));
  return check_launch("silu_mul");
}

int pdllm_rope_pages(void* k_cache, const int32_t* page_ids, int64_t start, int64_t n_tokens, const void* cos_tab,
                     const void* sin_tab, int page_size, int num_kv_heads, int head_dim, int dtype,
                     int64_t num_pages, int32_t* status, void* stream) {
  if (n_tokens < 0 || start < 0 || page_size <= 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0)
    return fail(PDLLM_E_INVALID, "rope_pages: bad sizes");
  if (n_tokens == 0) return 0;
  if (!k_cache || !page_ids || !cos_tab || !sin_tab) return fail(PDLLM_E_INVALID, "rope_pages: null pointer");
  const int grid = grid_for(n_tokens * num_kv_heads * (head_dim / 2), 256);
#define PDLLM_ROPE_LAUNCH(T)                                                                                        \
  rope_pages_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(static_cast<T*>(k_cache), page_ids, start, n_tokens,    \
                                                            static_cast<const T*>(cos_tab),                         \
                                                            static_cast<const T*>(sin_tab), page_size,              \
                                                            num_kv_heads, head_dim, num_pages, status)
  if (dtype == PDLLM_F32) PDLLM_ROPE_LAUNCH(float);
  else if (dtype == PDLLM_BF16) PDLLM_ROPE_LAUNCH(__nv_bfloat16);
  else if (dtype == PDLLM_F16) PDLLM_ROPE_LAUNCH(__half);
  else return fail(PDLLM_E_UNSUPPORTED, "rope_pages: dtype must be f32, bf16 or f16");
#undef PDLLM_ROPE_LAUNCH
  return check_launch("rope_pages");
}

int pdllm_copy_pages(const void* src_cache, const int32_t* src_page_ids, void* dst_cache, const int32_t* dst_page_ids,
                     int64_t n_lists, int64_t tokens_per_list, int page_size, int64_t row_elems, int elem_bytes,
                     int64_t src_num_pages, int64_t dst_num_pages, int32_t* status, void* stream) {
  if (n_lists < 0 || tokens_per_list < 0 || page_size <= 0 || row_elems <= 0) return fail(PDLLM_E_INVALID, "copy_pages: bad sizes");
  if (n_lists == 0 || tokens_per_list == 0) return 0;
  if (!src_cache || !dst_cache || !src_page_ids || !dst_page_ids) return fail(PDLLM_E_INVALID, "copy_pages: null pointer");
  if (tokens_per_list >= (1ll << 31)) return fail(PDLLM_E_INVALID, "copy_pages: list too long");
  const int64_t row_bytes = row_elems * elem_bytes;
  if (row_bytes % 16 != 0 || !aligned16(src_cache) || !aligned16(dst_cache)) return fail(PDLLM_E_UNSUPPORTED, "copy_pages: rows must be 16-byte multiples");
  const int segs = static_cast<int>(row_bytes / 16);
  const int64_t n_tokens = n_lists * tokens_per_list;
  page_to_page_kernel<<<grid_for(n_tokens * segs, 256), 256, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(src_cache), src_page_ids, static_cast<uint4*>(dst_cache), dst_page_ids, n_tokens,
      static_cast<int>(tokens_per_list), page_size, segs, src_num_pages, dst_num_pages, status);
  return check_launch("copy_pages");
}

int pdllm_enable_peer_access(int device, int peer_device) {
  if (device == peer_device) return 0;
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, device, peer_device);
  if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaDeviceCanAccessPeer: %s", cudaGetErrorString(e));
  if (!can) return fail(PDLLM_E_UNSUPPORTED, "device %d cannot map the memory of device %d", device, peer_device);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled) { cudaGetLastError(); return 0; }
  if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
  return 0;
}

int pdllm_compact_pages_per_head(void* cache, const int32_t* src_page_ids, const int32_t* dst_page_ids,
                                 const int64_t* keep, int64_t keep_count, int64_t src_tokens,
                                 int64_t dst_start, int64_t dst_tokens, int page_size, int num_kv_heads, int head_dim,
                                 int elem_bytes, int64_t num_pages, void* staging, int32_t* status,
                                 void* stream) {
  if (keep_count < 0 || page_size <= 0 || num_kv_heads <= 0 || head_dim <= 0 || dst_start < 0)
    return fail(PDLLM_E_INVALID, "compact_pages_per_head: bad sizes");
  if (keep_count == 0) return 0;
  if (dst_start + keep_count > dst_tokens)
    return fail(PDLLM_E_INVALID, "compact_pages_per_head: rows [%lld, %lld) do not fit the %lld tokens of dst_page_ids",
                (long long)dst_start, (long long)(dst_start + keep_count), (long long)dst_tokens);
  if (!cache || !src_page_ids || !dst_page_ids || !keep || !staging) return fail(PDLLM_E_INVALID, "compact_pages_per_head: null pointer");
  const int64_t head_bytes = static_cast<int64_t>(head_dim) * elem_bytes;
  if (head_bytes % 16 != 0 || !aligned16(cache) || !aligned16(staging)) return fail(PDLLM_E_UNSUPPORTED, "compact_pages_per_head: head rows must be 16-byte multiples");
  const int segs_per_head = static_cast<int>(head_bytes / 16);
  const int64_t per_tok = static_cast<int64_t>(num_kv_heads) * segs_per_head;
  const int grid = grid_for(keep_count * per_tok, 256);
  compact_gather_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const uint4*>(cache), src_page_ids, keep, keep_count, src_tokens,
                                                             page_size, num_kv_heads, segs_per_head, num_pages,
                                                             static_cast<uint4*>(staging), status);
  int rc = check_launch("compact_gather_kernel");
  if (rc != 0) return rc;
  compact_scatter_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<uint4*>(cache), dst_page_ids, keep_count, dst_start, page_size,
                                                              per_tok, num_pages, static_cast<const uint4*>(staging), status);
  return check_launch("compact_scatter_kernel");
}

// ------------------------------------------------------------------------------------------------ linear layers
int64_t pdllm_linear_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m < 0 || n < 0 || k < 0) return PDLLM_E_INVALID;
  return gemm::workspace_bytes(m, n, k);
}

int pdllm_linear(const void* x, int64_t x_stride, const void* weight, int64_t w_stride, const void* bias, void* out,
                 int64_t out_stride, int64_t m, int64_t n, int64_t k, int dtype, int epilogue, void* workspace,
                 int64_t workspace_bytes, int workspace_zeroed, int32_t* status, void* stream) {
  if (m < 0 || n <= 0 || k <= 0) return fail(PDLLM_E_INVALID, "linear: bad sizes m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
  if (m == 0) return 0;
  if (!x || !weight || !out) return fail(PDLLM_E_INVALID, "linear: null pointer");
  if (dtype != PDLLM_BF16 && dtype != PDLLM_F16) return fail(PDLLM_E_UNSUPPORTED, "linear: dtype must be bf16 or fp16 (tensor-core operands)");
  const int flags = epilogue;
  epilogue &= ~PDLLM_LINEAR_WEIGHTS_AT_REST;
  if (epilogue != PDLLM_EPI_NONE && epilogue != PDLLM_EPI_SILU_MUL) return fail(PDLLM_E_INVALID, "linear: unknown epilogue %d", epilogue);
  if (epilogue == PDLLM_EPI_SILU_MUL && (bias != nullptr || n % 2 != 0))
    return fail(PDLLM_E_INVALID, "linear: the SiLU-mul epilogue takes an even number of interleaved (gate, up) rows and no bias");
  const int64_t out_cols = epilogue == PDLLM_EPI_SILU_MUL ? n / 2 : n;
  if (k % 8 != 0 || x_stride % 8 != 0 || w_stride % 8 != 0 || x_stride < k || w_stride < k || out_stride < out_cols)
    return fail(PDLLM_E_UNSUPPORTED, "linear: K and the row strides of x and weight must be multiples of 8 elements (16 bytes)");
  if (!aligned16(x) || !aligned16(weight)) return fail(PDLLM_E_UNSUPPORTED, "linear: x and weight must be 16-byte aligned");
  if (m > 128 && (out_stride % 8 != 0 || !aligned16(out) || out_cols % 8 != 0))
    return fail(PDLLM_E_UNSUPPORTED, "linear: with more than 128 rows, out needs 16-byte aligned rows and a column count that is a multiple of 8");
  if (m >= (1ll << 31) || n >= (1ll << 31) || k >= (1ll << 31)) return fail(PDLLM_E_UNSUPPORTED, "linear: extent exceeds the tensor-map coordinate range");
  return gemm::launch(x, x_stride, weight, w_stride, bias, out, out_stride, m, n, k, dtype, epilogue | (flags & PDLLM_LINEAR_WEIGHTS_AT_REST), workspace, workspace_bytes,
                      workspace_zeroed, status, as_stream(stream));
}

}  // extern "C"
