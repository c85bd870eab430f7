// Row-wise pieces of the transformer block that sit between the GEMMs: RMSNorm (with the residual add in front of
// it), rotary embedding applied in place to the q and k slices of the fused QKV projection, and SiLU(gate) * up.
// All are HBM-bound: each reads and writes its rows once. In eager PyTorch each is 3 to 10 separate launches,
// which at 32 rows per denoise step cost more than the weights the step reads.
// Arithmetic follows the eager expressions of the model the reference vendors
// (prefilling_dllm_eval/model_cache/dream/model_dream.py:117-131 RMSNorm in fp32 then cast then scaled; :208-264
// rotate-half RoPE with tables cast to the model dtype; :277-278 SwiGLU): every intermediate that eager mode would
// materialise in the model dtype is rounded to it here as well.
#pragma once

#include "common.cuh"

namespace pdllm {

// out[t, :] = weight * round_T(x[t, :] * rsqrt(mean(x[t, :]^2) + eps)); when `delta` is given, first
// x[t, :] = round_T(x[t, :] + delta[t, :]) (the residual stream, updated in place). One CTA per row.
template <typename T>
__global__ void add_rmsnorm_kernel(T* __restrict__ x, const T* __restrict__ delta, const T* __restrict__ weight,
                                   T* __restrict__ out, int hidden, int64_t x_stride, int64_t delta_stride,
                                   int64_t out_stride, float eps) {
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();
  const int64_t row = blockIdx.x;
  T* xr = x + row * x_stride;
  const T* dr = delta ? delta + row * delta_stride : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = to_f32<T>(xr[i]);
    if (dr) {
      v = to_f32<T>(from_f32<T>(v + to_f32<T>(dr[i])));
      xr[i] = from_f32<T>(v);
    }
    ss += v * v;
  }
  __shared__ float partial[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? partial[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(partial[0] / static_cast<float>(hidden) + eps);
  T* orow = out + row * out_stride;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    // the row was just written by this same thread when delta != nullptr, so the re-read sees the updated value
    const float normed = to_f32<T>(from_f32<T>(to_f32<T>(xr[i]) * inv));
    orow[i] = from_f32<T>(to_f32<T>(weight[i]) * normed);
  }
}

// The same operation for 16-bit rows whose length is a multiple of 8 and at most 8 x blockDim: every thread owns ONE 16-byte
// vector of the row, loads x, delta and weight at once (three independent loads in flight instead of two dependent passes
// over global memory), keeps the updated row in registers across the reduction and writes x and out once. At decode shapes
// (a few dozen rows) the kernel is pure latency, and this form has one load round trip where the loop form has three.
template <typename T>
__global__ void add_rmsnorm_vec_kernel(T* __restrict__ x, const T* __restrict__ delta, const T* __restrict__ weight,
                                       T* __restrict__ out, int hidden, int64_t x_stride, int64_t delta_stride,
                                       int64_t out_stride, float eps) {
  const int64_t row = blockIdx.x;
  const int v0 = threadIdx.x * 8;
  const bool live = v0 < hidden;
  uint4 xv = make_uint4(0, 0, 0, 0), dv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
  if (live) wv = *reinterpret_cast<const uint4*>(weight + v0);     // never written by a kernel of the stream: may be read before the wait
  grid_dependency_wait();
  grid_launch_dependents();
  T* xr = x + row * x_stride;
  if (live) {
    xv = *reinterpret_cast<const uint4*>(xr + v0);
    if (delta != nullptr) dv = *reinterpret_cast<const uint4*>(delta + row * delta_stride + v0);
  }
  float v[8];
  {
    const T* xe = reinterpret_cast<const T*>(&xv);
    const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f = to_f32<T>(xe[i]);
      if (delta != nullptr) f = to_f32<T>(from_f32<T>(f + to_f32<T>(de[i])));
      v[i] = f;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  __shared__ float partial[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = (threadIdx.x & 31) < (blockDim.x >> 5) ? partial[threadIdx.x & 31] : 0.f;
  total = warp_sum(total);                       // every warp reduces the (at most 32) warp sums itself: no second barrier
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  if (live) {
    uint4 ov, nx;
    T* oe = reinterpret_cast<T*>(&ov);
    T* ne = reinterpret_cast<T*>(&nx);
    const T* we = reinterpret_cast<const T*>(&wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ne[i] = from_f32<T>(v[i]);
      const float normed = to_f32<T>(from_f32<T>(v[i] * inv));
      oe[i] = from_f32<T>(to_f32<T>(we[i]) * normed);
    }
    if (delta != nullptr) *reinterpret_cast<uint4*>(xr + v0) = nx;
    *reinterpret_cast<uint4*>(out + row * out_stride + v0) = ov;
  }
}

// x[t, h, :] = x * cos[t] + rotate_half(x) * sin[t] for the first `num_heads` heads of every row of a strided
// [T, *, D] buffer (q and k are adjacent head ranges of the fused projection output). One thread per (t, h, i < D/2).
template <typename T>
__global__ void rope_inplace_kernel(T* __restrict__ x, const T* __restrict__ cos_tab, const T* __restrict__ sin_tab,
                                    int64_t n_tokens, int num_heads, int head_dim, int64_t row_stride) {
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();
  const int half = head_dim / 2;
  const int64_t per_tok = static_cast<int64_t>(num_heads) * half;
  const int64_t total = n_tokens * per_tok;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / per_tok;
    const int rem = static_cast<int>(idx - t * per_tok);
    const int h = rem / half, i = rem - h * half;
    T* row = x + t * row_stride + static_cast<int64_t>(h) * head_dim;
    const T* c = cos_tab + t * head_dim;
    const T* s = sin_tab + t * head_dim;
    const float x1 = to_f32<T>(row[i]), x2 = to_f32<T>(row[i + half]);
    const float a1 = to_f32<T>(from_f32<T>(__fmul_rn(x1, to_f32<T>(c[i]))));
    const float b1 = to_f32<T>(from_f32<T>(__fmul_rn(-x2, to_f32<T>(s[i]))));
    const float a2 = to_f32<T>(from_f32<T>(__fmul_rn(x2, to_f32<T>(c[i + half]))));
    const float b2 = to_f32<T>(from_f32<T>(__fmul_rn(x1, to_f32<T>(s[i + half]))));
    row[i] = from_f32<T>(__fadd_rn(a1, b1));
    row[i + half] = from_f32<T>(__fadd_rn(a2, b2));
  }
}

// RoPE of the q and k heads of a fused [T, Hq + 2 Hkv, D] projection output AND the page write of its k and v heads, in one
// launch for 16-bit rows: a thread owns the two 16-byte vectors [8j, 8j + 8) and [D/2 + 8j, D/2 + 8j + 8) of one head of one
// token — the pairs the rotation combines — with the rounding of rope_inplace_kernel; k heads go to k_cache[slot] after the
// rotation (or before it, k_before_rotation: per-head eviction assigns positions after compaction), v heads are copied to
// v_cache[slot]. slot < 0 (or no slot_mapping) skips the write; slot >= num_slots is reported and skipped.
template <typename T>
__global__ void rope_store_kernel(T* __restrict__ qkv, const T* __restrict__ cos_tab, const T* __restrict__ sin_tab, int64_t n_tokens,
                                  int hq, int hkv, int head_dim, int64_t row_stride, T* __restrict__ k_cache, T* __restrict__ v_cache,
                                  const int32_t* __restrict__ slot_mapping, int64_t num_slots, int k_before_rotation, int32_t* status) {
  grid_dependency_wait();     // launched ahead of its predecessor's end: nothing global is touched before this
  grid_launch_dependents();
  const int half = head_dim / 2, vecs = half / 8, heads = hq + 2 * hkv;
  const int64_t total = n_tokens * heads * vecs;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % vecs);
    const int h = static_cast<int>((idx / vecs) % heads);
    const int64_t t = idx / (static_cast<int64_t>(vecs) * heads);
    T* row = qkv + t * row_stride + static_cast<int64_t>(h) * head_dim;
    uint4 lo = *reinterpret_cast<const uint4*>(row + 8 * j);
    uint4 hi = *reinterpret_cast<const uint4*>(row + half + 8 * j);
    const bool is_v = h >= hq + hkv, is_k = h >= hq && !is_v;
    int64_t slot = -1;
    if ((is_k || is_v) && slot_mapping != nullptr) {
      slot = slot_mapping[t];
      if (slot >= num_slots) {
        if (j == 0) report_status(status, PDLLM_S_BAD_SLOT);
        slot = -1;
      }
    }
    if (is_v) {
      if (slot >= 0) {
        T* dst = v_cache + (slot * hkv + (h - hq - hkv)) * head_dim;
        *reinterpret_cast<uint4*>(dst + 8 * j) = lo;
        *reinterpret_cast<uint4*>(dst + half + 8 * j) = hi;
      }
      continue;
    }
    const uint4 c_lo = *reinterpret_cast<const uint4*>(cos_tab + t * head_dim + 8 * j);
    const uint4 c_hi = *reinterpret_cast<const uint4*>(cos_tab + t * head_dim + half + 8 * j);
    const uint4 s_lo = *reinterpret_cast<const uint4*>(sin_tab + t * head_dim + 8 * j);
    const uint4 s_hi = *reinterpret_cast<const uint4*>(sin_tab + t * head_dim + half + 8 * j);
    T* kdst = (is_k && slot >= 0) ? k_cache + (slot * hkv + (h - hq)) * head_dim : nullptr;
    if (kdst != nullptr && k_before_rotation) {
      *reinterpret_cast<uint4*>(kdst + 8 * j) = lo;
      *reinterpret_cast<uint4*>(kdst + half + 8 * j) = hi;
    }
    uint4 o_lo, o_hi;
    {
      const T* x1 = reinterpret_cast<const T*>(&lo);
      const T* x2 = reinterpret_cast<const T*>(&hi);
      const T* c1 = reinterpret_cast<const T*>(&c_lo);
      const T* c2 = reinterpret_cast<const T*>(&c_hi);
      const T* s1 = reinterpret_cast<const T*>(&s_lo);
      const T* s2 = reinterpret_cast<const T*>(&s_hi);
      T* r1 = reinterpret_cast<T*>(&o_lo);
      T* r2 = reinterpret_cast<T*>(&o_hi);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float a = to_f32<T>(x1[i]), b = to_f32<T>(x2[i]);
        const float a1 = to_f32<T>(from_f32<T>(__fmul_rn(a, to_f32<T>(c1[i]))));
        const float b1 = to_f32<T>(from_f32<T>(__fmul_rn(-b, to_f32<T>(s1[i]))));
        const float a2 = to_f32<T>(from_f32<T>(__fmul_rn(b, to_f32<T>(c2[i]))));
        const float b2 = to_f32<T>(from_f32<T>(__fmul_rn(a, to_f32<T>(s2[i]))));
        r1[i] = from_f32<T>(__fadd_rn(a1, b1));
        r2[i] = from_f32<T>(__fadd_rn(a2, b2));
      }
    }
    *reinterpret_cast<uint4*>(row + 8 * j) = o_lo;
    *reinterpret_cast<uint4*>(row + half + 8 * j) = o_hi;
    if (kdst != nullptr && !k_before_rotation) {
      *reinterpret_cast<uint4*>(kdst + 8 * j) = o_lo;
      *reinterpret_cast<uint4*>(kdst + half + 8 * j) = o_hi;
    }
  }
}

// out[t, i] = round_T(silu(gate[t, i])) * up[t, i] with gate = gu[t, :inter], up = gu[t, inter:]
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t n_tokens, int inter,
                                int64_t gu_stride, int64_t out_stride) {
  const int64_t total = n_tokens * inter;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = idx / inter;
    const int i = static_cast<int>(idx - t * inter);
    const float g = to_f32<T>(gu[t * gu_stride + i]);
    const float u = to_f32<T>(gu[t * gu_stride + inter + i]);
    const float act = to_f32<T>(from_f32<T>(g / (1.f + expf(-g))));
    out[t * out_stride + i] = from_f32<T>(act * u);
  }
}

}  // namespace pdllm
