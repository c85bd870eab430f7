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
