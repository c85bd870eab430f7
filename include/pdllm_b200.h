/*
 * pdllm_b200 — C-ABI of the B200 (sm_100a) kernels behind the Prefilling-dLLM long-context hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*), launches on that
 * stream without synchronising, and returns an int status:
 *      0            success (kernel(s) enqueued)
 *     <0            argument rejected on the host (PDLLM_E_*); pdllm_last_error() has the message
 *     >0            a cudaError_t raised by the launch
 * Index-carrying device inputs (slot mappings, block tables, label ids) are range-checked ON the device:
 * a bad entry is skipped and, when the caller passed a `status` word, its PDLLM_S_* code is atomically
 * max-ed into it. Nothing here traps, asserts or spins without a bound.
 *
 * The reference project is pure Python (Triton/Flex kernels); it has no FFI. Each declaration below
 * names the reference Python op (file:line within that project) whose job it takes over. The Python shims
 * with the reference's exact signatures live in prefilling-dllm_b200/ops.py and bind this header by ctypes.
 */
#ifndef PDLLM_B200_H_
#define PDLLM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PDLLM_ABI_VERSION 5

/* element types of floating-point tensors */
#define PDLLM_F32 0
#define PDLLM_BF16 1
#define PDLLM_F16 2

/* host-side argument errors */
#define PDLLM_E_INVALID (-1)     /* null pointer, negative size, unsupported combination */
#define PDLLM_E_UNSUPPORTED (-2) /* valid in the reference but not built here (fp8 KV, alibi, sliding window) */
#define PDLLM_E_WORKSPACE (-3)   /* workspace missing or too small */
#define PDLLM_E_DRIVER (-4)      /* tensor-map encode entry point unavailable */

/* device status word codes (larger = more severe; the word keeps the max seen) */
#define PDLLM_S_OK 0
#define PDLLM_S_BAD_SLOT 1    /* slot_mapping entry >= num_slots (entry skipped) */
#define PDLLM_S_BAD_PAGE 2    /* block_table entry outside [0, num_pages) (page treated as page 0, keys masked) */
#define PDLLM_S_BAD_LABEL 3   /* label id outside [0, vocab) (row scored as -inf) */
#define PDLLM_S_BAD_INDEX 4   /* keep / gather index out of range (entry skipped) */
#define PDLLM_S_WAIT_TIMEOUT 8 /* a bounded mbarrier wait expired; output of that launch is invalid */

int pdllm_abi_version(void);
const char* pdllm_last_error(void);
/* 1 when the current device is compute capability 10.x (tcgen05/TMA paths usable), else 0; <0 on error */
int pdllm_device_supported(void);

/* ------------------------------------------------------------------------------------------------
 * (5) KV page writes
 * replaces store_kvcache_unified_layout / store_kvcache_kernel_diffusion_lm
 *   prefilling_dllm_engine/prefilling_dllm/layers/attention/ops/kv_cache_kernels.py:34-55, 150-172
 * key/value: [n_tokens, Hkv*D] rows with row strides key_stride/value_stride (elements);
 * k_cache/v_cache: [num_slots, Hkv*D] (= [pages, page_size, Hkv, D] flattened); slot < 0 skips the token.
 * ---------------------------------------------------------------------------------------------- */
int pdllm_store_kvcache_unified(const void* key, const void* value, void* k_cache, void* v_cache,
                                const int32_t* slot_mapping, int64_t n_tokens, int64_t row_elems,
                                int64_t key_stride, int64_t value_stride, int elem_bytes,
                                int64_t num_slots, int32_t* status, void* stream);

/* replaces store_kvcache_distinct_layout / store_kvcache_kernel_diffusion_lm_distinct
 *   .../ops/kv_cache_kernels.py:58-147
 * k_cache: [pages, Hkv, D/x, page_size, x], v_cache: [pages, Hkv, D, page_size], both contiguous. */
int pdllm_store_kvcache_distinct(const void* key, const void* value, void* k_cache, void* v_cache,
                                 const int32_t* slot_mapping, int64_t n_tokens, int num_kv_heads,
                                 int head_dim, int page_size, int x, int64_t key_stride,
                                 int64_t value_stride, int elem_bytes, int64_t num_pages,
                                 int32_t* status, void* stream);

/* replaces load_kvcache / load_kvcache_kernel_kv (the per-layer gather the fused decode kernel removes;
 * kept because the reference's op table exports it)
 *   .../ops/kv_cache_kernels.py:175-327
 * Writes, per sequence s, rows [cu_seqlens_k[s], +ctx_len[s]) from the pages of block_table[s] and then the
 * seq_lens[s] new rows. k_out/v_out: [total_k, Hkv, D] contiguous. */
int pdllm_load_kvcache(const void* k_cache, const void* v_cache, const void* k_new, const void* v_new,
                       const int32_t* block_table, int64_t block_table_stride, int max_pages,
                       const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                       const int32_t* context_lens, int num_seqs, int num_kv_heads, int head_dim,
                       int page_size, int64_t num_pages, int64_t new_stride, int elem_bytes,
                       void* k_out, void* v_out, int64_t total_k, int32_t* status, void* stream);

/* ------------------------------------------------------------------------------------------------
 * (3)+(1) block-table attention: new rows attend [selected prefix pages ‖ new rows]
 * replaces chunked_prefill_paged_decode → context_attention_fwd → _fwd_kernel_d2f
 *   .../ops/chunked_prefill_decoding_unified_kernel.py:220-274, .../ops/prefix_prefill.py:25-230, 1046-1080
 * and the unified-layout path load_kvcache + flex_attention of
 *   prefilling_dllm_engine/prefilling_dllm/layers/attention/attention_v4.py:359-397
 * ---------------------------------------------------------------------------------------------- */
#define PDLLM_KV_NONE 0     /* no cached context (prefill of new rows only) */
#define PDLLM_KV_UNIFIED 1  /* k/v cache [pages, page_size, Hkv, D] */
#define PDLLM_KV_DISTINCT 2 /* k [pages, Hkv, D/x, page_size, x], v [pages, Hkv, D, page_size] */

#define PDLLM_MASK_BLOCK 0  /* reference d2f rule: key n visible to row m iff n < q_len and
                               (bidirectional or n < (m / (2*diffusion_blk) + 1) * 2*diffusion_blk), and mask[m,n] */
#define PDLLM_MASK_CAUSAL 1 /* key n visible to row m iff n <= m (sequence-local), context always visible */

#define PDLLM_ATTN_AUTO 0   /* tcgen05 kernel when the shape allows, else the SIMT kernel */
#define PDLLM_ATTN_SIMT 1   /* force the fp32-accumulating SIMT kernel */
#define PDLLM_ATTN_TC 2     /* force the tcgen05/TMEM kernel; PDLLM_E_UNSUPPORTED if the shape does not allow */

typedef struct pdllm_attn_params {
  const void* q;      /* [total_q, Hq, D], row stride q_stride elements, heads contiguous */
  const void* k_new;  /* [total_q, Hkv, D] */
  const void* v_new;  /* [total_q, Hkv, D] */
  void* out;          /* [total_q, Hq, D] */
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_table;   /* [num_seqs, max_pages] page ids in ANY order */
  const int32_t* cu_seqlens_q;  /* [num_seqs + 1] */
  const int32_t* seq_lens;      /* [num_seqs] context + new rows (the reference's b_seq_len) */
  const uint8_t* mask;          /* optional bool mask over new rows x new keys, sequence-LOCAL indices */
  int32_t* status;              /* optional device status word */
  void* workspace;              /* split-KV arrival counters + partials; pdllm_attn_workspace_bytes(); 256-byte aligned */
  void* trace;                  /* profiling aid of the tcgen05 kernel, read only by a library built with
                                   -DPDLLM_ENABLE_TRACE (the release build ignores it): int64 [8 CTAs][64 iterations]
                                   [16 events] of clock64() timestamps, zero-initialised by the caller; NULL = off */
  int64_t workspace_bytes;
  int64_t q_stride, k_stride, v_stride, out_stride; /* row strides, elements */
  int64_t block_table_stride;
  int64_t mask_stride_m, mask_stride_n;
  int64_t num_pages;
  int64_t total_q;
  int32_t num_seqs, max_pages;
  int32_t num_q_heads, num_kv_heads, head_dim;
  int32_t page_size, x;        /* x: inner pack of the distinct K layout */
  int32_t kv_layout;           /* PDLLM_KV_* */
  int32_t dtype;               /* PDLLM_F32 / BF16 / F16 (q, k, v, caches and out share it) */
  int32_t mask_mode;           /* PDLLM_MASK_* */
  int32_t bidirectional;
  int32_t diffusion_blk;
  int32_t max_query_len, max_seq_len; /* host-known upper bounds used for grid sizing */
  int32_t impl;                /* PDLLM_ATTN_* */
  int32_t num_splits;          /* 0 = choose; >=1 forces the KV split count of the tcgen05 kernel */
  float sm_scale;
  int32_t workspace_zeroed;    /* non-zero: the caller zero-filled `workspace` once and after any launch that raised
                                  PDLLM_S_WAIT_TIMEOUT; the split-KV arrival counters in its first 64 KB are then known to
                                  be zero (every launch returns them to zero) and no memset is enqueued. 0 = clear them */
} pdllm_attn_params;

int64_t pdllm_attn_workspace_bytes(const pdllm_attn_params* p);
int pdllm_paged_attention(const pdllm_attn_params* p, void* stream);
/* which kernel pdllm_paged_attention would run for p: PDLLM_ATTN_SIMT or PDLLM_ATTN_TC (<0 = error) */
int pdllm_attn_select_impl(const pdllm_attn_params* p);
/* 1 when the tcgen05 path would take its few-rows form for p (one query tile per CTA, the KV splits of a (sequence, KV head,
 * query tile) merged inside a thread-block cluster through distributed shared memory: a block of decode rows of one or a few
 * requests, the shape of attention_v4.py:375-397 per layer per denoise step), 0 when the twin-tile form, <0 = error */
int pdllm_attn_uses_cluster_kernel(const pdllm_attn_params* p);

/* ------------------------------------------------------------------------------------------------
 * (4) confidence-threshold unmask step
 * replaces _shift_logits + sample_tokens + the top-k/threshold loop of
 *   prefilling_dllm_eval/fastdllm_parallelcomp.py:204-233, 1007-1015, 2399-2441
 *   prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:1648-1681, 2133-2157
 * logits: [block_len, vocab] rows of the block forward; row r of the SHIFTED view is logits[r-1] for r>=1
 * and last_logit for r==0 when shift != 0 (Dream); shift == 0 uses logits[r] (LLaDA).
 * block_ids (int64, in place): every slot equal to mask_id is a candidate; the most confident candidate is
 * always filled, every other candidate is filled iff conf >= threshold. conf_dtype says in which type the
 * reference rounds the softmax probability (and the threshold) before comparing: PDLLM_F32 for the engine,
 * the logits dtype for the eval path. Greedy (temperature 0) only.
 * out_counts[0] = candidates before the step, out_counts[1] = slots filled, out_counts[2] = candidates left.
 * out_conf (optional, fp32 [block_len]) / out_x0 (optional, int64 [block_len]) expose per-slot results.
 * workspace: pdllm_unmask_workspace_bytes(block_len) bytes, zero-initialised ONCE by the caller (the kernel
 * leaves it zeroed again).
 * ---------------------------------------------------------------------------------------------- */
int64_t pdllm_unmask_workspace_bytes(int block_len);
int pdllm_unmask_step(const void* logits, int64_t logits_stride, const void* last_logit, int dtype,
                      int block_len, int64_t vocab, int shift, int64_t* block_ids, int64_t mask_id,
                      float threshold, int conf_dtype, int32_t* out_counts, float* out_conf,
                      int64_t* out_x0, void* workspace, int64_t workspace_bytes, void* stream);

/* The same step for `batch` blocks in ONE launch (requests that share a denoise step, as the engine's decode of
 * several sequences does, fastdllm_engine.py:2133-2157 run per sequence there). Request z reads logits rows at
 * logits + z * batch_stride (elements), its last logit at last_logit + z * last_stride, its ids at
 * block_ids + z * block_len; out_counts is [batch][3], out_conf / out_x0 are [batch][block_len]; the workspace holds
 * batch * pdllm_unmask_workspace_bytes(block_len) bytes, zero-initialised once by the caller. batch <= 65535. */
int pdllm_unmask_step_batched(const void* logits, int64_t logits_stride, int64_t batch_stride, const void* last_logit,
                              int64_t last_stride, int dtype, int batch, int block_len, int64_t vocab, int shift,
                              int64_t* block_ids, int64_t mask_id, float threshold, int conf_dtype,
                              int32_t* out_counts, float* out_conf, int64_t* out_x0, void* workspace,
                              int64_t workspace_bytes, void* stream);

/* Same step as pdllm_unmask_step, for callers that cannot hand over device scratch. It has no counterpart in the
 * reference. Some hosts of the decode loop have given every byte of device memory they may use to the KV page pool
 * and run the loop under a rule of "no allocation after start-up" (an allocation there can fail, and cudaMalloc
 * stalls the whole device while it runs); others sit behind an interface that carries only inputs and outputs.
 * For them the partial-reduction scratch lives inside the library: a fixed array of about 7 KB that every GPU which
 * loads the library holds until the process exits, enough for block_len <= PDLLM_UNMASK_STATIC_MAX_BLOCK; longer
 * blocks are refused with PDLLM_E_INVALID. The call allocates nothing. The first call on a device looks up the
 * array's device address (a one-time set-up; make that first call before any stream capture begins). All calls share
 * the one array and it keeps the previous call's contents: the entry point clears the words that must start at zero,
 * and two calls whose kernels overlap on the GPU (different streams, no ordering between them) race on it — issue
 * them on one stream or order them with events. */
#define PDLLM_UNMASK_STATIC_MAX_BLOCK 64
int pdllm_unmask_step_static(const void* logits, int64_t logits_stride, const void* last_logit, int dtype,
                             int block_len, int64_t vocab, int shift, int64_t* block_ids, int64_t mask_id,
                             float threshold, int conf_dtype, int32_t* out_counts, float* out_conf,
                             int64_t* out_x0, void* stream);

/* ------------------------------------------------------------------------------------------------
 * (2a) draft-self-information score tail
 * replaces index_select(label_pos-1) → log_softmax(fp32) → gather(labels) → −mean NLL
 *   prefilling_dllm_eval/fastdllm_parallelcomp.py:1415-1422 (engine twin fastdllm_engine.py:1147-1152)
 * rows: [n_chunks * n_labels, vocab] logits rows ALREADY gathered at label_pos-1 (row = chunk*n_labels+i);
 * labels: [n_labels] int64 shared by all chunks. scores_out: [n_chunks] fp32; non-finite → -inf.
 * nll_out (optional): [n_chunks * n_labels] fp32 per-label NLL.
 * ---------------------------------------------------------------------------------------------- */
int pdllm_self_information_scores(const void* rows, int64_t row_stride, int dtype, int n_chunks,
                                  int n_labels, int64_t vocab, const int64_t* labels,
                                  float* scores_out, float* nll_out, int32_t* status, void* stream);

/* (2b) stable top-K of chunk scores
 * replaces sorted(remaining, key=score, reverse=True)[:topk] then ascending order
 *   prefilling_dllm_eval/fastdllm_parallelcomp.py:1949-1953 (engine fastdllm_engine.py:1200-1204)
 * Ties keep the lower chunk index; keep_first forces chunk 0 outside the K budget; topk <= 0 selects all.
 * selected_out: [n_chunks] int32 ascending, first *count_out entries valid. n_chunks <= 1024. */
int pdllm_topk_chunks(const float* scores, int n_chunks, int topk, int keep_first,
                      int32_t* selected_out, int32_t* count_out, void* stream);

/* (2c) query→chunk attention mass for intra-chunk eviction
 * replaces query_to_chunk_attention_scores (_query_max_den_kernel + _query_to_chunk_scores_kernel)
 *   .../ops/triton_eviction_scorer.py:6-210
 * and _chunk_attention_head_scores of prefilling_dllm_eval/fastdllm_parallelcomp.py:1639-1667
 * q: [L, Hq, D], k: [L, Hkv, D] (rotated), rows prefix_len+chunk_len .. +query_len are the query window.
 * out: fp32 [Hq, chunk_len] = sum (or mean) over the window rows of softmax(q·k*scale)[chunk columns];
 * causal != 0 hides keys after the row. workspace: pdllm_evict_workspace_bytes(Hq, query_len, L). */
int64_t pdllm_evict_workspace_bytes(int num_q_heads, int query_len, int64_t key_len);
int pdllm_query_to_chunk_scores(const void* q, const void* k, int dtype, int64_t key_len,
                                int num_q_heads, int num_kv_heads, int head_dim, int prefix_len,
                                int chunk_len, int query_len, float scale, int reduce_mean, int causal,
                                float* out, void* workspace, int64_t workspace_bytes, void* stream);

/* (2c) pooled scores → kept positions
 * replaces max_pool1d(k, pad k/2, stride 1) + head/group reduction + _select_positions_from_token_scores
 *   prefilling_dllm_eval/fastdllm_parallelcomp.py:1607-1626, 1754-1760, 1997-2023
 *   prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:904-927, 1396-1432
 * head_scores: fp32 [n_layers, Hq, chunk_len]. pool_kernel <= 1 disables pooling.
 * granularity 0 (global): per layer sum over heads, mean over layers → ONE row of chunk_len scores →
 *   keep_out [1, keep_count]. granularity 1 (per_head): per layer, mean over the query heads of each KV
 *   group → keep_out [n_layers, Hkv, keep_count].
 * force_first != 0 keeps position 0 and picks keep_count-1 from 1..chunk_len-1; largest != 0 keeps the
 * highest scores. Ties keep the lower position. Output positions are ascending int64.
 * pooled_out (optional): fp32 rows actually ranked ([1, chunk_len] or [n_layers, Hkv, chunk_len]). */
int pdllm_evict_select(const float* head_scores, int n_layers, int num_q_heads, int num_kv_heads,
                       int chunk_len, int pool_kernel, int granularity, int keep_count, int force_first,
                       int largest, int64_t* keep_out, float* pooled_out, void* stream);

/* ------------------------------------------------------------------------------------------------
 * KV movement on the prefill/decode boundary
 * replaces the advanced-index gathers/scatters of _snapshot_prompt_cache_per_layer /
 * _load_prompt_cache_per_layer / _compact_prompt_cache_per_layer_per_head /
 * make_pd_record_from_remote_engine
 *   prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:607-698, 800-859
 * All caches are unified layout [pages, page_size, Hkv, D].
 * ---------------------------------------------------------------------------------------------- */
/* pages → dense: out[t, :] = cache[page_ids[t / page_size], t % page_size, :] for t < n_tokens */
int pdllm_gather_pages(const void* cache, const int32_t* page_ids, int64_t n_tokens, int page_size,
                       int64_t row_elems, int elem_bytes, int64_t num_pages, void* out,
                       int32_t* status, void* stream);
/* dense → pages (inverse of the above) */
int pdllm_scatter_pages(const void* src, const int32_t* page_ids, int64_t n_tokens, int page_size,
                        int64_t row_elems, int elem_bytes, int64_t num_pages, void* cache,
                        int32_t* status, void* stream);
/* pool -> pool: for each of n_lists page lists (one per layer and K/V plane, `ceil(tokens_per_list / page_size)` ids
 * each, concatenated) copy the first tokens_per_list tokens of the src pages into the dst pages. src_cache may be the
 * pool of ANOTHER GPU mapped by peer access (pdllm_enable_peer_access): the kernel, launched on the destination GPU,
 * then reads it across NVLink with plain loads — no staging copy. Both id lists are read by the kernel on the
 * launching device. Replaces the per-layer gather / .to() / scatter of make_pd_record_from_remote_engine
 *   prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:845-859 */
int pdllm_copy_pages(const void* src_cache, const int32_t* src_page_ids, void* dst_cache, const int32_t* dst_page_ids,
                     int64_t n_lists, int64_t tokens_per_list, int page_size, int64_t row_elems, int elem_bytes,
                     int64_t src_num_pages, int64_t dst_num_pages, int32_t* status, void* stream);
/* map peer_device's memory into device's address space (idempotent); PDLLM_E_UNSUPPORTED if the GPUs have no peer path */
int pdllm_enable_peer_access(int device, int peer_device);
/* per-(KV head) compaction: dst token dst_start + j of head h := src token keep[h, j]; src and dst page lists may be
 * the same pages (in-place compaction to the front): the kernel stages through `staging`
 * ([keep_count, Hkv, D] elements) so overlapping ranges are safe. src_tokens / dst_tokens: tokens covered by the
 * two page lists (list length x page_size, or fewer); rows outside them are refused, not written. */
int pdllm_compact_pages_per_head(void* cache, const int32_t* src_page_ids, const int32_t* dst_page_ids,
                                 const int64_t* keep, int64_t keep_count, int64_t src_tokens,
                                 int64_t dst_start, int64_t dst_tokens, int page_size, int num_kv_heads, int head_dim,
                                 int elem_bytes, int64_t num_pages, void* staging, int32_t* status,
                                 void* stream);

/* Rotary embedding of K rows that are already in pages and were stored UN-rotated: tokens [start, start + n_tokens)
 * of the page list, every KV head, in place; cos_tab / sin_tab are [n_tokens, head_dim] in the cache dtype (the
 * model's own tables: cat(freqs, freqs)). Arithmetic rounds each product and the sum to the cache dtype, like the
 * eager `k * cos + rotate_half(k) * sin`.
 * Serves the eval class's per-head eviction, whose model caches un-rotated keys and rotates them at read time
 * with the COMPACTED positions (kept row j of every head gets chunk_positions[j], not its original position):
 *   prefilling_dllm_eval/fastdllm_parallelcomp.py:1076-1125 (_gather_cache_per_layer_per_head), :2284-2288,
 *   :2890-2912 (active_positions_after_prefill). */
int pdllm_rope_pages(void* k_cache, const int32_t* page_ids, int64_t start, int64_t n_tokens, const void* cos_tab,
                     const void* sin_tab, int page_size, int num_kv_heads, int head_dim, int dtype,
                     int64_t num_pages, int32_t* status, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Row-wise pieces of the transformer block between the GEMMs (one launch each instead of 3-10 eager ones)
 * replaces RMSNorm.rms_forward / add_rms_forward   prefilling_dllm_engine/prefilling_dllm/layers/layernorm.py:18-41
 *          apply_rotary_emb / RotaryEmbedding.forward  .../layers/rotary_embedding.py:6-65
 *          SiluAndMul.forward                          .../layers/activation.py:12-14
 * with the rounding of the eval model the reference vendors (prefilling_dllm_eval/model_cache/dream/model_dream.py
 * :117-131, :208-264, :277-278): every intermediate eager mode would hold in the model dtype is rounded to it.
 * ---------------------------------------------------------------------------------------------- */
/* if delta != NULL: x[t,:] += delta[t,:] (in place); then out[t,:] = weight * dtype(x[t,:] * rsqrt(mean(x^2) + eps)) */
int pdllm_add_rmsnorm(void* x, const void* delta, const void* weight, void* out, int64_t n_tokens, int hidden, int64_t x_stride,
                      int64_t delta_stride, int64_t out_stride, float eps, int dtype, void* stream);
/* rotate the first num_heads heads of every row of x [n_tokens, *, head_dim] (row stride in elements) in place;
 * cos_tab / sin_tab: [n_tokens, head_dim] in the same dtype (cat(freqs, freqs) layout) */
int pdllm_rope_inplace(void* x, const void* cos_tab, const void* sin_tab, int64_t n_tokens, int num_heads, int head_dim,
                       int64_t row_stride, int dtype, void* stream);
/* RoPE of the q and k heads of a fused projection output qkv [n_tokens, num_q_heads + 2 num_kv_heads, head_dim] (row stride in
 * elements) in place AND the page write of its k and v heads, one launch (bf16 / fp16, head_dim a multiple of 16):
 * replaces the pair  q, k = self.rotary_emb(positions, q, k)          prefilling_dllm_engine/prefilling_dllm/models/dream.py:75-76
 *                    store_kvcache_unified_layout(k, v, k_cache, ...)  .../layers/attention/attention_v4.py:330-331
 * k_cache / v_cache: this layer's unified pools [num_slots, num_kv_heads, head_dim]; slot_mapping [n_tokens] int32 (slot < 0:
 * not stored; NULL with NULL caches: rotation only). k_before_rotation != 0 stores the k rows as projected (un-rotated). */
int pdllm_rope_store(void* qkv, int64_t row_stride, const void* cos_tab, const void* sin_tab, int64_t n_tokens, int num_q_heads,
                     int num_kv_heads, int head_dim, void* k_cache, void* v_cache, const int32_t* slot_mapping, int64_t num_slots,
                     int k_before_rotation, int dtype, int32_t* status, void* stream);
/* out[t, i] = dtype(silu(gate_up[t, i])) * gate_up[t, inter + i] */
int pdllm_silu_mul(const void* gate_up, void* out, int64_t n_tokens, int inter, int64_t gu_stride, int64_t out_stride, int dtype,
                   void* stream);

/* ------------------------------------------------------------------------------------------------
 * Linear layers of the transformer block on the tensor cores: out[m, n] = x[m, k] . weight[n, k]^T (+ bias[n])
 * replaces QKVParallelLinear / MergedColumnParallelLinear / RowParallelLinear.forward (F.linear)
 *            prefilling_dllm_engine/prefilling_dllm/layers/linear.py:108-244
 *          ParallelLMHead.forward                      .../layers/embed_head.py:63-74
 *          SiluAndMul.forward fused behind gate_up_proj .../layers/activation.py:12-14, models/dream.py:130-136
 * x: [m, k] rows with stride x_stride, weight: [n, k] rows with stride w_stride (the nn.Linear layout), out: [m, n] rows
 * with stride out_stride (all in elements); bf16 or fp16, fp32 accumulation, the result rounded once to the dtype.
 * epilogue PDLLM_EPI_SILU_MUL: the weight rows are INTERLEAVED (row 2i = gate_i, row 2i + 1 = up_i) and
 *   out[m, i] = dtype(silu(dtype(gate_i))) * dtype(up_i), out is [m, n / 2]; no bias.
 * Up to 128 rows the weights are streamed once from HBM with the k-blocks dealt evenly over all SMs (stream-K); that
 * path needs pdllm_linear_workspace_bytes() of workspace whose first 64 KB hold arrival counters: zero-fill it once and
 * pass workspace_zeroed != 0 (the kernel returns every counter to zero), or pass 0 and a memset is enqueued first.
 * PDLLM_LINEAR_WEIGHTS_AT_REST, OR-ed into `epilogue`: the caller vouches that nothing still in flight on the stream writes
 *   `weight` (model weights after loading); the kernel may then start streaming weights while the kernel before it on the
 *   stream is still finishing (programmatic dependent launch) and reads x, bias and the workspace only afterwards.
 */
#define PDLLM_EPI_NONE 0
#define PDLLM_EPI_SILU_MUL 1
#define PDLLM_LINEAR_WEIGHTS_AT_REST 0x100
int64_t pdllm_linear_workspace_bytes(int64_t m, int64_t n, int64_t k);
int pdllm_linear(const void* x, int64_t x_stride, const void* weight, int64_t w_stride, const void* bias, void* out,
                 int64_t out_stride, int64_t m, int64_t n, int64_t k, int dtype, int epilogue, void* workspace,
                 int64_t workspace_bytes, int workspace_zeroed, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* PDLLM_B200_H_ */
