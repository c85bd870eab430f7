// Scoring-side kernels: the fused confidence-threshold unmask step, the self-information score tail, the
// stable top-K over chunk scores, the query->chunk attention mass and the pooled keep-position selection.
// All vocabulary / key sweeps are single-pass HBM-bound reductions in fp32.
#pragma once

#include "common.cuh"

namespace pdllm {

// =====================================================================================================
// (4) unmask step
// =====================================================================================================
constexpr int kUnmaskThreads = 256;
constexpr int kUnmaskChunks = 8;   // CTAs per logits row, so 32 rows x 8 = 256 CTAs keep every SM pulling HBM
constexpr int kUnmaskMaxBlock = 1024;

struct UnmaskWs {             // layout of the caller's workspace, all 4-byte words
  // float  pmax [block_len][kUnmaskChunks]
  // float  psum [block_len][kUnmaskChunks]
  // int    pidx [block_len][kUnmaskChunks]
  // float  conf [block_len]
  // int    x0   [block_len]
  // uint   row_counter [block_len]   (zero on entry, zero on exit)
  // uint   done_counter              (zero on entry, zero on exit)
};

__host__ __device__ inline int64_t unmask_ws_words(int block_len) {
  return static_cast<int64_t>(block_len) * (3 * kUnmaskChunks + 3) + 1;
}

template <typename T>
__device__ __forceinline__ const T* unmask_row_ptr(const T* logits, int64_t stride, const T* last_logit, int shift, int r) {
  if (!shift) return logits + static_cast<int64_t>(r) * stride;
  if (r == 0) return last_logit != nullptr ? last_logit : logits;  // no last logit: the reference copies row 0
  return logits + static_cast<int64_t>(r - 1) * stride;
}

template <typename T>
__global__ void __launch_bounds__(kUnmaskThreads)
unmask_kernel(const T* __restrict__ logits, int64_t stride, const T* __restrict__ last_logit, int block_len,
              int64_t vocab, int shift, int64_t* __restrict__ block_ids, int64_t mask_id, float threshold,
              int conf_dtype, int32_t* __restrict__ out_counts, float* __restrict__ out_conf,
              int64_t* __restrict__ out_x0, float* __restrict__ ws, int64_t batch_stride, int64_t last_stride) {
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();
  // blockIdx.z: one block of slots per request, each with its own logits rows, ids, outputs and scratch
  {
    const int64_t z = blockIdx.z;
    logits += z * batch_stride;
    if (last_logit != nullptr) last_logit += z * last_stride;
    block_ids += z * block_len;
    if (out_counts != nullptr) out_counts += z * 3;
    if (out_conf != nullptr) out_conf += z * block_len;
    if (out_x0 != nullptr) out_x0 += z * block_len;
    ws += z * unmask_ws_words(block_len);
  }
  float* pmax = ws;
  float* psum = pmax + block_len * kUnmaskChunks;
  int* pidx = reinterpret_cast<int*>(psum + block_len * kUnmaskChunks);
  float* conf = reinterpret_cast<float*>(pidx + block_len * kUnmaskChunks);
  int* x0 = reinterpret_cast<int*>(conf + block_len);
  unsigned* row_counter = reinterpret_cast<unsigned*>(x0 + block_len);
  unsigned* done_counter = row_counter + block_len;

  __shared__ float s_max[kUnmaskThreads / 32];
  __shared__ float s_sum[kUnmaskThreads / 32];
  __shared__ int s_idx[kUnmaskThreads / 32];
  __shared__ int s_flag;
  __shared__ float s_rowM, s_rowS;

  const int r = blockIdx.y;
  const int chunk = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool masked = block_ids[r] == mask_id;
  const T* row = unmask_row_ptr(logits, stride, last_logit, shift, r);

  // ---- phase 1: (max, first argmax, sum exp) of this CTA's slice of the row ----
  if (masked) {
    const int64_t per = (vocab + kUnmaskChunks - 1) / kUnmaskChunks;
    // 16-byte aligned slices so the vector loads stay aligned (rows are 16-byte aligned when stride % VEC == 0)
    constexpr int VEC = Vec16<T>::N;
    const int64_t per_al = (per + VEC - 1) / VEC * VEC;
    const int64_t b = min(vocab, chunk * per_al), e = min(vocab, b + per_al);
    const bool aligned = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
    float mx = -INFINITY; int ix = 0x7fffffff; float sm = 0.f;
    auto feed = [&](float x, int64_t i) {
      if (x > mx) { sm = sm * expf(mx - x) + 1.f; mx = x; ix = static_cast<int>(i); }
      else if (x == mx) { sm += 1.f; if (i < ix) ix = static_cast<int>(i); }
      else sm += expf(x - mx);
    };
    // One rescale per 16-byte vector instead of one branch and one exp call per element. A thread meets its indices in
    // ascending order, so a strict '>' keeps the first occurrence of its maximum.
    auto feed_vec = [&](const float* f, int64_t base) {
      float vm = f[0];
#pragma unroll
      for (int j = 1; j < VEC; ++j) vm = fmaxf(vm, f[j]);
      if (vm > mx) {
        sm = (mx == -INFINITY) ? 0.f : sm * __expf(mx - vm);
        mx = vm;
        int first = VEC - 1;
#pragma unroll
        for (int j = VEC - 2; j >= 0; --j) first = (f[j] == vm) ? j : first;
        ix = static_cast<int>(base) + first;
      }
      if (mx > -INFINITY) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) sm += __expf(f[j] - mx);   // arguments <= 0
      }
    };
    if (aligned) {
      const int64_t nvec = (e - b) / VEC;
      constexpr int kInFlight = 4;   // a CTA streams 38 KB of a row: keep four 16-byte loads per thread in flight
      int64_t vI = tid;
      for (; vI + (kInFlight - 1) * kUnmaskThreads < nvec; vI += kInFlight * kUnmaskThreads) {
        float f[kInFlight][VEC];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) Vec16<T>::load(row + b + (vI + u * kUnmaskThreads) * VEC, f[u]);
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) feed_vec(f[u], b + (vI + u * kUnmaskThreads) * VEC);
      }
      for (; vI < nvec; vI += kUnmaskThreads) {
        float f[VEC];
        Vec16<T>::load(row + b + vI * VEC, f);
        feed_vec(f, b + vI * VEC);
      }
      for (int64_t i = b + nvec * VEC + tid; i < e; i += kUnmaskThreads) feed(to_f32<T>(row[i]), i);
    } else {
      for (int64_t i = b + tid; i < e; i += kUnmaskThreads) feed(to_f32<T>(row[i]), i);
    }
    // combine lanes: larger max wins, ties keep the lower index, sums rescaled to the winner
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float omx = __shfl_xor_sync(0xffffffffu, mx, o);
      const float osm = __shfl_xor_sync(0xffffffffu, sm, o);
      const int oix = __shfl_xor_sync(0xffffffffu, ix, o);
      const float nm = fmaxf(mx, omx);
      const float a = (mx == -INFINITY) ? 0.f : sm * expf(mx - nm);
      const float c = (omx == -INFINITY) ? 0.f : osm * expf(omx - nm);
      if (omx > mx || (omx == mx && oix < ix)) ix = oix;
      mx = nm; sm = a + c;
    }
    if (lane == 0) { s_max[warp] = mx; s_sum[warp] = sm; s_idx[warp] = ix; }
    __syncthreads();
    if (tid == 0) {
      float M = s_max[0], S = s_sum[0]; int I = s_idx[0];
      for (int w = 1; w < kUnmaskThreads / 32; ++w) {
        const float nm = fmaxf(M, s_max[w]);
        const float a = (M == -INFINITY) ? 0.f : S * expf(M - nm);
        const float c = (s_max[w] == -INFINITY) ? 0.f : s_sum[w] * expf(s_max[w] - nm);
        if (s_max[w] > M || (s_max[w] == M && s_idx[w] < I)) I = s_idx[w];
        M = nm; S = a + c;
      }
      pmax[r * kUnmaskChunks + chunk] = M; psum[r * kUnmaskChunks + chunk] = S; pidx[r * kUnmaskChunks + chunk] = I;
    }
  }

  // ---- phase 2: the last CTA of a row finalises it ----
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&row_counter[r], 1u);
    s_flag = (prev == kUnmaskChunks - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();

  if (masked) {
    if (tid == 0) {
      float M = -INFINITY, S = 0.f; int I = 0x7fffffff;
      for (int c = 0; c < kUnmaskChunks; ++c) {
        const float cm = pmax[r * kUnmaskChunks + c], cs = psum[r * kUnmaskChunks + c]; const int ci = pidx[r * kUnmaskChunks + c];
        if (cm == -INFINITY) continue;
        const float nm = fmaxf(M, cm);
        const float a = (M == -INFINITY) ? 0.f : S * expf(M - nm);
        const float cc = cs * expf(cm - nm);
        if (cm > M || (cm == M && ci < I)) I = ci;
        M = nm; S = a + cc;
      }
      s_rowM = M; s_rowS = S;
      conf[r] = round_through(1.f / S, conf_dtype);  // softmax probability of the arg-max, in the reference's dtype
      x0[r] = I;
    }
    __syncthreads();
    if (conf_dtype != PDLLM_F32) {
      // The reference takes max/argmax over probabilities already rounded to the model dtype, so every token
      // whose rounded probability equals the rounded maximum ties with it and the lowest index wins.
      const float M = s_rowM, S = s_rowS, target = conf[r];
      int first = 0x7fffffff;
      // Only logits within a hair of the maximum can round to the maximum's probability (bf16 / fp16 keep 8 / 11 significant
      // bits: ratio > 1 - 2^-7, i.e. a logit gap under 0.008): compare first, evaluate the exponential for those few only.
      const float floor_x = M - 0.03f;
      constexpr int VEC = Vec16<T>::N;
      if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        const int64_t nvec = vocab / VEC;
        for (int64_t vI = tid; vI < nvec && first == 0x7fffffff; vI += kUnmaskThreads) {
          float f[VEC];
          Vec16<T>::load(row + vI * VEC, f);
#pragma unroll
          for (int j = VEC - 1; j >= 0; --j) {
            if (f[j] >= floor_x && round_through(expf(f[j] - M) / S, conf_dtype) == target) first = static_cast<int>(vI * VEC + j);
          }
        }
        for (int64_t i = nvec * VEC + tid; i < vocab; i += kUnmaskThreads) {
          const float x = to_f32<T>(row[i]);
          if (x >= floor_x && round_through(expf(x - M) / S, conf_dtype) == target) first = min(first, static_cast<int>(i));
        }
      } else {
        for (int64_t i = tid; i < vocab; i += kUnmaskThreads) {
          const float x = to_f32<T>(row[i]);
          if (x >= floor_x && round_through(expf(x - M) / S, conf_dtype) == target) { first = static_cast<int>(i); break; }  // i ascends per thread
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
      if (lane == 0) s_idx[warp] = first;
      __syncthreads();
      if (tid == 0) {
        int f = s_idx[0];
        for (int w = 1; w < kUnmaskThreads / 32; ++w) f = min(f, s_idx[w]);
        if (f != 0x7fffffff) x0[r] = f;
      }
    }
  }
  __syncthreads();

  // ---- phase 3: the last row to finish applies the accept rule ----
  if (tid == 0) {
    row_counter[r] = 0;
    __threadfence();
    const unsigned prev = atomicAdd(done_counter, 1u);
    s_flag = (prev == static_cast<unsigned>(block_len) - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();

  __shared__ float s_best;
  __shared__ int s_besti;
  __shared__ int s_cnt[3];
  if (tid == 0) { s_cnt[0] = 0; s_cnt[1] = 0; s_cnt[2] = 0; }
  __syncthreads();
  // most confident candidate (ties: lowest slot)
  float best = -INFINITY; int besti = 0x7fffffff;
  for (int i = tid; i < block_len; i += kUnmaskThreads) {
    if (block_ids[i] == mask_id) {
      const float c = conf[i];
      if (c > best || (c == best && i < besti) || besti == 0x7fffffff) { best = c; besti = i; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (oi != 0x7fffffff && (besti == 0x7fffffff || ob > best || (ob == best && oi < besti))) { best = ob; besti = oi; }
  }
  if (lane == 0) { s_max[warp] = best; s_idx[warp] = besti; }
  __syncthreads();
  if (tid == 0) {
    float b = s_max[0]; int bi = s_idx[0];
    for (int w = 1; w < kUnmaskThreads / 32; ++w) {
      if (s_idx[w] != 0x7fffffff && (bi == 0x7fffffff || s_max[w] > b || (s_max[w] == b && s_idx[w] < bi))) { b = s_max[w]; bi = s_idx[w]; }
    }
    s_best = b; s_besti = bi;
  }
  __syncthreads();
  const float thr = round_through(threshold, conf_dtype);
  const int top = s_besti;
  for (int i = tid; i < block_len; i += kUnmaskThreads) {
    const bool cand = block_ids[i] == mask_id;
    if (out_conf) out_conf[i] = cand ? conf[i] : -INFINITY;
    if (out_x0) out_x0[i] = cand ? static_cast<int64_t>(x0[i]) : block_ids[i];
    if (cand) {
      atomicAdd(&s_cnt[0], 1);
      if (i == top || conf[i] >= thr) { block_ids[i] = x0[i]; atomicAdd(&s_cnt[1], 1); }
    }
  }
  __syncthreads();
  if (tid == 0) {
    if (out_counts) { out_counts[0] = s_cnt[0]; out_counts[1] = s_cnt[1]; out_counts[2] = s_cnt[0] - s_cnt[1]; }
    *done_counter = 0;
  }
}

// =====================================================================================================
// (2a) self-information tail
// =====================================================================================================
constexpr int kScoreThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kScoreThreads)
self_info_nll_kernel(const T* __restrict__ rows, int64_t row_stride, int n_labels, int64_t vocab,
                     const int64_t* __restrict__ labels, float* __restrict__ nll, int32_t* status) {
  const int64_t ridx = blockIdx.x;
  const T* row = rows + ridx * row_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float s_m[kScoreThreads / 32], s_s[kScoreThreads / 32];
  constexpr int VEC = Vec16<T>::N;
  float mx = -INFINITY, sm = 0.f;
  auto feed = [&](float x) {
    if (x > mx) { sm = sm * expf(mx - x) + 1.f; mx = x; } else if (mx > -INFINITY) sm += expf(x - mx);
  };
  // one rescale per 16-byte vector instead of one branch per element
  auto feed_vec = [&](const float* f) {
    float vm = f[0];
#pragma unroll
    for (int j = 1; j < VEC; ++j) vm = fmaxf(vm, f[j]);
    if (vm > mx) { sm *= expf(mx - vm); mx = vm; }
    if (mx > -INFINITY) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) sm += __expf(f[j] - mx);   // arguments <= 0; 2^-21 relative error, far inside the 1e-4 the scores are held to
    }
  };
  if ((reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const int64_t nvec = vocab / VEC;
    // four 16-byte loads in flight per thread: one row is 300 KB and a CTA streams it alone
    constexpr int kInFlight = 4;
    int64_t v = tid;
    for (; v + (kInFlight - 1) * kScoreThreads < nvec; v += kInFlight * kScoreThreads) {
      float f[kInFlight][VEC];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) Vec16<T>::load(row + (v + u * kScoreThreads) * VEC, f[u]);
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) feed_vec(f[u]);
    }
    for (; v < nvec; v += kScoreThreads) {
      float f[VEC];
      Vec16<T>::load(row + v * VEC, f);
      feed_vec(f);
    }
    for (int64_t i = nvec * VEC + tid; i < vocab; i += kScoreThreads) feed(to_f32<T>(row[i]));
  } else {
    for (int64_t i = tid; i < vocab; i += kScoreThreads) feed(to_f32<T>(row[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
    const float nm = fmaxf(mx, om);
    const float a = (mx == -INFINITY) ? 0.f : sm * expf(mx - nm);
    const float c = (om == -INFINITY) ? 0.f : os * expf(om - nm);
    mx = nm; sm = a + c;
  }
  if (lane == 0) { s_m[warp] = mx; s_s[warp] = sm; }
  __syncthreads();
  if (tid == 0) {
    float M = s_m[0], S = s_s[0];
    for (int w = 1; w < kScoreThreads / 32; ++w) {
      const float nm = fmaxf(M, s_m[w]);
      const float a = (M == -INFINITY) ? 0.f : S * expf(M - nm);
      const float c = (s_m[w] == -INFINITY) ? 0.f : s_s[w] * expf(s_m[w] - nm);
      M = nm; S = a + c;
    }
    const int64_t label = labels[ridx % n_labels];
    if (label < 0 || label >= vocab) {
      report_status(status, PDLLM_S_BAD_LABEL);
      nll[ridx] = INFINITY;
    } else {
      // log_softmax(x)[label] = x - max - log(sum exp(x - max))
      nll[ridx] = -((to_f32<T>(row[label]) - M) - logf(S));
    }
  }
}

// score[c] = -mean_i nll[c, i]; non-finite becomes -inf (the reference's isfinite filter)
__global__ void self_info_mean_kernel(const float* __restrict__ nll, int n_chunks, int n_labels, float* __restrict__ scores) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chunks) return;
  double acc = 0.0;
  for (int i = 0; i < n_labels; ++i) acc += static_cast<double>(nll[static_cast<int64_t>(c) * n_labels + i]);
  const float s = n_labels > 0 ? static_cast<float>(-(acc / n_labels)) : -INFINITY;
  scores[c] = isfinite(s) ? s : -INFINITY;
}

// =====================================================================================================
// (2b) stable top-K of chunk scores
// =====================================================================================================
__global__ void topk_chunks_kernel(const float* __restrict__ scores, int n, int topk, int keep_first,
                                   int32_t* __restrict__ selected, int32_t* __restrict__ count) {
  __shared__ float s[1024];
  __shared__ int flag[1024];
  const int i = threadIdx.x;
  if (i < n) { const float v = scores[i]; s[i] = isfinite(v) ? v : -INFINITY; }
  __syncthreads();
  const int forced = (keep_first && n > 0) ? 1 : 0;
  const int remaining = n - forced;
  const int k = (topk <= 0) ? remaining : min(topk, remaining);
  int sel = 0;
  if (i < n) {
    if (forced && i == 0) sel = 1;
    else {
      // rank among the non-forced chunks under (score descending, index ascending) = Python's stable sort
      int rank = 0;
      for (int j = forced; j < n; ++j) {
        if (j == i) continue;
        if (s[j] > s[i] || (s[j] == s[i] && j < i)) ++rank;
      }
      sel = rank < k ? 1 : 0;
    }
    flag[i] = sel;
  }
  __syncthreads();
  if (i < n && sel) {
    int pos = 0;
    for (int j = 0; j < i; ++j) pos += flag[j];
    selected[pos] = i;
  }
  if (i == 0) {
    int c = 0;
    for (int j = 0; j < n; ++j) c += flag[j];
    *count = c;
  }
}

// =====================================================================================================
// (2c) query -> chunk attention mass
// =====================================================================================================
constexpr int kEvictKeys = 64;     // keys per CTA in the logits pass
constexpr int kEvictThreads = 256;

// logits[h, qi, n] = scale * <q[row_qi, h], k[n, kvh]>, -inf where causal hides key n from row_qi
template <typename T>
__global__ void __launch_bounds__(kEvictThreads)
evict_logits_kernel(const T* __restrict__ q, const T* __restrict__ k, int64_t key_len, int num_q_heads,
                    int num_kv_heads, int head_dim, int query_start, int query_len, float scale, int causal,
                    float* __restrict__ logits) {
  extern __shared__ float sh[];
  float* sk = sh;                                         // [kEvictKeys][head_dim + 1]
  float* sq = sh + kEvictKeys * (head_dim + 1);           // [query_len][head_dim]
  const int h = blockIdx.y;
  const int kvh = h / (num_q_heads / num_kv_heads);
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kEvictKeys;
  const int tid = threadIdx.x;
  for (int i = tid; i < kEvictKeys * head_dim; i += kEvictThreads) {
    const int kr = i / head_dim, d = i - kr * head_dim;
    const int64_t n = n0 + kr;
    sk[kr * (head_dim + 1) + d] = (n < key_len) ? to_f32<T>(k[(n * num_kv_heads + kvh) * head_dim + d]) : 0.f;
  }
  for (int i = tid; i < query_len * head_dim; i += kEvictThreads) {
    const int qi = i / head_dim, d = i - qi * head_dim;
    sq[i] = to_f32<T>(q[(static_cast<int64_t>(query_start + qi) * num_q_heads + h) * head_dim + d]);
  }
  __syncthreads();
  const int kr = tid % kEvictKeys;
  const int64_t n = n0 + kr;
  for (int qi = tid / kEvictKeys; qi < query_len; qi += kEvictThreads / kEvictKeys) {
    float dot = 0.f;
    const float* kp = sk + kr * (head_dim + 1);
    const float* qp = sq + qi * head_dim;
    for (int d = 0; d < head_dim; ++d) dot = fmaf(kp[d], qp[d], dot);
    float v = dot * scale;
    if (causal && n > query_start + qi) v = -INFINITY;
    if (n < key_len) logits[(static_cast<int64_t>(h) * query_len + qi) * key_len + n] = v;
  }
}

// out[h, c] = sum_qi softmax(logits[h, qi, :])[prefix_len + c]   (optionally / query_len)
__global__ void __launch_bounds__(kEvictThreads)
evict_reduce_kernel(const float* __restrict__ logits, int64_t key_len, int query_len, int prefix_len, int chunk_len,
                    int reduce_mean, float* __restrict__ out) {
  extern __shared__ float sh[];
  float* s_m = sh;               // [query_len]
  float* s_d = sh + query_len;   // [query_len]
  __shared__ float red[kEvictThreads / 32];
  const int h = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int qi = 0; qi < query_len; ++qi) {
    const float* row = logits + (static_cast<int64_t>(h) * query_len + qi) * key_len;
    float mx = -INFINITY;
    for (int64_t n = tid; n < key_len; n += kEvictThreads) mx = fmaxf(mx, row[n]);
    mx = warp_max(mx);
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) { float M = red[0]; for (int w = 1; w < kEvictThreads / 32; ++w) M = fmaxf(M, red[w]); s_m[qi] = M; }
    __syncthreads();
    const float M = s_m[qi];
    float sm = 0.f;
    for (int64_t n = tid; n < key_len; n += kEvictThreads) sm += expf(row[n] - M);
    sm = warp_sum(sm);
    if (lane == 0) red[warp] = sm;
    __syncthreads();
    if (tid == 0) { float S = 0.f; for (int w = 0; w < kEvictThreads / 32; ++w) S += red[w]; s_d[qi] = S; }
    __syncthreads();
  }
  for (int c = tid; c < chunk_len; c += kEvictThreads) {
    float acc = 0.f;
    for (int qi = 0; qi < query_len; ++qi) {
      const float l = logits[(static_cast<int64_t>(h) * query_len + qi) * key_len + prefix_len + c];
      acc += expf(l - s_m[qi]) / s_d[qi];
    }
    if (reduce_mean) acc /= static_cast<float>(query_len);
    out[static_cast<int64_t>(h) * chunk_len + c] = acc;
  }
}

// =====================================================================================================
// (2c) pooled scores -> kept positions. One CTA per output row.
// =====================================================================================================
constexpr int kSelectThreads = 1024;

__device__ __forceinline__ float pooled_at(const float* row, int c, int chunk_len, int pool_kernel) {
  if (pool_kernel <= 1) return row[c];
  const int kernel = min(pool_kernel, chunk_len);
  const int pad = kernel / 2;
  float m = -INFINITY;
  for (int j = c - pad; j < c - pad + kernel; ++j) {
    if (j >= 0 && j < chunk_len) m = fmaxf(m, row[j]);
  }
  return m;
}

__global__ void __launch_bounds__(kSelectThreads)
evict_select_kernel(const float* __restrict__ head_scores, int n_layers, int num_q_heads, int num_kv_heads,
                    int chunk_len, int pool_kernel, int granularity, int keep_count, int force_first, int largest,
                    int64_t* __restrict__ keep_out, float* __restrict__ pooled_out) {
  extern __shared__ float sc[];                 // [chunk_len] scores of this row
  int* flags = reinterpret_cast<int*>(sc + chunk_len);  // [chunk_len]
  __shared__ int s_block[kSelectThreads / 32];
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int G = num_q_heads / num_kv_heads;

  // ---- scores of this row ----
  for (int c = tid; c < chunk_len; c += kSelectThreads) {
    float v;
    if (granularity == 0) {
      // per layer: sum over heads of the pooled head scores; then mean over layers
      float lsum = 0.f;
      for (int l = 0; l < n_layers; ++l) {
        float hs = 0.f;
        for (int h = 0; h < num_q_heads; ++h) {
          hs += pooled_at(head_scores + (static_cast<int64_t>(l) * num_q_heads + h) * chunk_len, c, chunk_len, pool_kernel);
        }
        lsum += hs;
      }
      v = lsum / static_cast<float>(n_layers);
    } else {
      const int l = row / num_kv_heads, kvh = row - l * num_kv_heads;
      float gs = 0.f;
      for (int g = 0; g < G; ++g) {
        gs += pooled_at(head_scores + (static_cast<int64_t>(l) * num_q_heads + kvh * G + g) * chunk_len, c, chunk_len, pool_kernel);
      }
      v = gs / static_cast<float>(G);
    }
    sc[c] = v;
    if (pooled_out) pooled_out[static_cast<int64_t>(row) * chunk_len + c] = v;
  }
  __syncthreads();

  // ---- selection by rank counting under (score desc|asc, position asc) ----
  const int first_cand = force_first ? 1 : 0;
  const int n_cand = chunk_len - first_cand;
  int k = keep_count - first_cand;
  if (k > n_cand) k = n_cand;
  if (k < 0) k = 0;
  for (int c = tid; c < chunk_len; c += kSelectThreads) {
    int sel;
    if (c < first_cand) sel = 1;
    else if (k >= n_cand) sel = 1;
    else {
      const float v = sc[c];
      int rank = 0;
      for (int j = first_cand; j < chunk_len; ++j) {
        const float o = sc[j];
        const bool before = largest ? (o > v) : (o < v);
        if (before || (o == v && j < c)) ++rank;
      }
      sel = rank < k ? 1 : 0;
    }
    flags[c] = sel;
  }
  __syncthreads();

  // ---- ordered compaction: exclusive prefix over flags ----
  // each thread owns a contiguous span so the output stays ascending
  const int per = (chunk_len + kSelectThreads - 1) / kSelectThreads;
  const int b = tid * per, e = min(chunk_len, b + per);
  int local = 0;
  for (int c = b; c < e; ++c) local += flags[c];
  // block exclusive scan of `local`
  const int lane = tid & 31, warp = tid >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_block[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_block[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    s_block[lane] = w;
  }
  __syncthreads();
  int pos = incl - local + (warp > 0 ? s_block[warp - 1] : 0);
  int64_t* dst = keep_out + static_cast<int64_t>(row) * keep_count;
  for (int c = b; c < e; ++c) {
    if (flags[c]) { if (pos < keep_count) dst[pos] = c; ++pos; }
  }
}

}  // namespace pdllm
