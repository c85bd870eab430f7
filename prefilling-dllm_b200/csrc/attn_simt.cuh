// Block-table attention, SIMT path: fp32 accumulation for any dtype (fp32 / bf16 / fp16), head_dim a
// multiple of 32 up to 256, both cache layouts, every mask rule. One warp owns one (new row, query head)
// pair and streams the keys with an online softmax. It is the full-precision path (fp32 models) and the
// on-device cross-check for the tcgen05 kernel; the tcgen05 kernel is the fast path.
#pragma once

#include "common.cuh"

namespace pdllm {

struct AttnSimtArgs {
  const void* q; const void* k_new; const void* v_new; void* out;
  const void* k_cache; const void* v_cache;
  const int32_t* block_table; const int32_t* cu_seqlens_q; const int32_t* seq_lens;
  const uint8_t* mask; int32_t* status;
  int64_t q_stride, k_stride, v_stride, out_stride, block_table_stride, mask_stride_m, mask_stride_n;
  int64_t num_pages, total_q;
  int num_seqs, max_pages, num_q_heads, num_kv_heads, head_dim, page_size, x, kv_layout;
  int mask_mode, bidirectional, block_m;  // block_m = 2 * diffusion_blk
  float sm_scale;
};

// visibility of new key n for new row m (both sequence-local)
__device__ __forceinline__ bool new_key_visible(const AttnSimtArgs& a, int m, int n, int q_len) {
  if (n >= q_len) return false;
  if (a.mask_mode == PDLLM_MASK_CAUSAL) return n <= m;
  if (!a.bidirectional && n >= (m / a.block_m + 1) * a.block_m) return false;
  if (a.mask != nullptr && a.mask[m * a.mask_stride_m + n * a.mask_stride_n] == 0) return false;
  return true;
}

template <typename T, int DPL>  // DPL = head_dim / 32 elements per lane (lane owns d = lane + 32*i)
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnSimtArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t total_pairs = a.total_q * a.num_q_heads;
  if (warp_global >= total_pairs) return;
  const int64_t row = warp_global / a.num_q_heads;
  const int head = static_cast<int>(warp_global - row * a.num_q_heads);
  const int group = a.num_q_heads / a.num_kv_heads;
  const int kvh = head / group;
  const int D = a.head_dim;

  // sequence owning this row
  int lo = 0, hi = a.num_seqs - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (a.cu_seqlens_q[mid] <= row) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int q_start = a.cu_seqlens_q[s];
  const int q_len = a.cu_seqlens_q[s + 1] - q_start;
  const int m = static_cast<int>(row - q_start);
  T* out_row = reinterpret_cast<T*>(a.out) + row * a.out_stride + static_cast<int64_t>(head) * D;
  if (m >= q_len) return;
  int ctx_len = 0;  // seq_lens may be null when there is no cache
  if (a.kv_layout != PDLLM_KV_NONE) ctx_len = max(0, a.seq_lens[s] - q_len);

  const T* q_row = reinterpret_cast<const T*>(a.q) + row * a.q_stride + static_cast<int64_t>(head) * D;
  float qv[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) qv[i] = to_f32<T>(q_row[lane + 32 * i]) * a.sm_scale;

  float m_run = -INFINITY, l_run = 0.f;
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;

  const T* kc = reinterpret_cast<const T*>(a.k_cache);
  const T* vc = reinterpret_cast<const T*>(a.v_cache);
  const int Hkv = a.num_kv_heads;

  // ---- context keys, page by page in block-table order ----
  for (int n0 = 0; n0 < ctx_len; n0 += a.page_size) {
    int pidx = n0 / a.page_size;
    int64_t page = (pidx < a.max_pages) ? a.block_table[s * a.block_table_stride + pidx] : -1;
    int n_in_page = min(a.page_size, ctx_len - n0);
    if (page < 0 || page >= a.num_pages) {
      if (lane == 0) report_status(a.status, PDLLM_S_BAD_PAGE);
      continue;  // keys of an unreadable page are masked out
    }
    for (int off = 0; off < n_in_page; ++off) {
      float kf[DPL], vf[DPL];
      if (a.kv_layout == PDLLM_KV_UNIFIED) {
        const T* kr = kc + ((page * a.page_size + off) * Hkv + kvh) * D;
        const T* vr = vc + ((page * a.page_size + off) * Hkv + kvh) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) { kf[i] = to_f32<T>(kr[lane + 32 * i]); vf[i] = to_f32<T>(vr[lane + 32 * i]); }
      } else {
        const int64_t page_elems = static_cast<int64_t>(Hkv) * D * a.page_size;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          int d = lane + 32 * i;
          int64_t koff = page * page_elems + (static_cast<int64_t>(kvh) * (D / a.x) + d / a.x) * a.page_size * a.x +
                         static_cast<int64_t>(off) * a.x + (d % a.x);
          int64_t voff = page * page_elems + (static_cast<int64_t>(kvh) * D + d) * a.page_size + off;
          kf[i] = to_f32<T>(kc[koff]); vf[i] = to_f32<T>(vc[voff]);
        }
      }
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) dot = fmaf(qv[i], kf[i], dot);
      dot = warp_sum(dot);
      float m_new = fmaxf(m_run, dot);
      float alpha = expf(m_run - m_new);
      float p = expf(dot - m_new);
      l_run = l_run * alpha + p;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = fmaf(p, vf[i], acc[i] * alpha);
      m_run = m_new;
    }
  }

  // ---- new keys of the same sequence ----
  const T* kn = reinterpret_cast<const T*>(a.k_new);
  const T* vn = reinterpret_cast<const T*>(a.v_new);
  int n_end = q_len;
  if (a.mask_mode == PDLLM_MASK_CAUSAL) n_end = m + 1;
  else if (!a.bidirectional) n_end = min(q_len, (m / a.block_m + 1) * a.block_m);
  for (int n = 0; n < n_end; ++n) {
    if (!new_key_visible(a, m, n, q_len)) continue;
    const T* kr = kn + (static_cast<int64_t>(q_start) + n) * a.k_stride + static_cast<int64_t>(kvh) * D;
    const T* vr = vn + (static_cast<int64_t>(q_start) + n) * a.v_stride + static_cast<int64_t>(kvh) * D;
    float dot = 0.f;
    float vf[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) { dot = fmaf(qv[i], to_f32<T>(kr[lane + 32 * i]), dot); vf[i] = to_f32<T>(vr[lane + 32 * i]); }
    dot = warp_sum(dot);
    float m_new = fmaxf(m_run, dot);
    float alpha = expf(m_run - m_new);
    float p = expf(dot - m_new);
    l_run = l_run * alpha + p;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = fmaf(p, vf[i], acc[i] * alpha);
    m_run = m_new;
  }

  // A row that sees no key at all: the reference divides 0 by its initial l=1 and writes zeros.
  float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) out_row[lane + 32 * i] = from_f32<T>(acc[i] * inv);
}

template <typename T>
int launch_attn_simt_t(const AttnSimtArgs& a, cudaStream_t stream) {
  int64_t pairs = a.total_q * a.num_q_heads;
  if (pairs == 0) return 0;
  int threads = 128;
  int64_t blocks = (pairs * 32 + threads - 1) / threads;
  switch (a.head_dim / 32) {
    case 1: attn_simt_kernel<T, 1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a); break;
    case 2: attn_simt_kernel<T, 2><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a); break;
    case 3: attn_simt_kernel<T, 3><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a); break;
    case 4: attn_simt_kernel<T, 4><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a); break;
    case 8: attn_simt_kernel<T, 8><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(a); break;
    default: return fail(PDLLM_E_UNSUPPORTED, "SIMT attention: head_dim %d not in {32,64,96,128,256}", a.head_dim);
  }
  return check_launch("attn_simt_kernel");
}

inline int launch_attn_simt(const pdllm_attn_params* p, cudaStream_t stream) {
  AttnSimtArgs a;
  a.q = p->q; a.k_new = p->k_new; a.v_new = p->v_new; a.out = p->out;
  a.k_cache = p->k_cache; a.v_cache = p->v_cache;
  a.block_table = p->block_table; a.cu_seqlens_q = p->cu_seqlens_q; a.seq_lens = p->seq_lens;
  a.mask = p->mask; a.status = p->status;
  a.q_stride = p->q_stride; a.k_stride = p->k_stride; a.v_stride = p->v_stride; a.out_stride = p->out_stride;
  a.block_table_stride = p->block_table_stride; a.mask_stride_m = p->mask_stride_m; a.mask_stride_n = p->mask_stride_n;
  a.num_pages = p->num_pages; a.total_q = p->total_q;
  a.num_seqs = p->num_seqs; a.max_pages = p->max_pages; a.num_q_heads = p->num_q_heads;
  a.num_kv_heads = p->num_kv_heads; a.head_dim = p->head_dim; a.page_size = p->page_size; a.x = p->x > 0 ? p->x : 1;
  a.kv_layout = p->kv_layout; a.mask_mode = p->mask_mode; a.bidirectional = p->bidirectional;
  a.block_m = 2 * (p->diffusion_blk > 0 ? p->diffusion_blk : 32);
  a.sm_scale = p->sm_scale;
  if (p->head_dim % 32 != 0 || p->head_dim > 256) {
    return fail(PDLLM_E_UNSUPPORTED, "SIMT attention needs head_dim %% 32 == 0 and <= 256, got %d", p->head_dim);
  }
  switch (p->dtype) {
    case PDLLM_F32: return launch_attn_simt_t<float>(a, stream);
    case PDLLM_BF16: return launch_attn_simt_t<__nv_bfloat16>(a, stream);
    case PDLLM_F16: return launch_attn_simt_t<__half>(a, stream);
    default: return fail(PDLLM_E_INVALID, "unknown dtype %d", p->dtype);
  }
}

}  // namespace pdllm
