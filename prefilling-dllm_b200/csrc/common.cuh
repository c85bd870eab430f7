// Shared helpers for the pdllm_b200 kernels: error plumbing, dtype loads, warp/block reductions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <utility>

#include "../../include/pdllm_b200.h"

namespace pdllm {

// ---- host-side error string (thread local, read through pdllm_last_error) -------------------------
inline std::string& last_error_ref() {
  static thread_local std::string s;
  return s;
}

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error_ref() = buf;
  return code;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(static_cast<int>(e), "%s: %s", what, cudaGetErrorString(e));
  }
  return 0;
}

// ---- device helpers --------------------------------------------------------------------------------
__device__ __forceinline__ void report_status(int32_t* status, int32_t code) {
  if (status != nullptr) atomicMax(status, code);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Round an fp32 value through `dtype` (PDLLM_F32/BF16/F16) and back, as torch does when a probability is
// materialised in the model dtype before a comparison.
__device__ __forceinline__ float round_through(float v, int dtype) {
  if (dtype == PDLLM_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == PDLLM_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 16-byte vector of 8 bf16/fp16 or 4 fp32 → fp32 array
template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* out) {
    float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  }
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* out) {
    uint4 v = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      out[2 * i] = f.x; out[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Vec16<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float* out) {
    uint4 v = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      out[2 * i] = f.x; out[2 * i + 1] = f.y;
    }
  }
};

// ---- programmatic dependent launch ----------------------------------------------------------------------------------
// The kernels of a forward run back to back on one stream, each a few microseconds long at decode shapes, so the gap between
// a kernel's last CTA and the next kernel's first instruction is a visible share of a step. A kernel launched with the
// programmatic-serialization attribute may be scheduled while its predecessor still runs; it does its on-chip set-up
// (barriers, TMEM allocation, descriptor prefetch), then calls grid_dependency_wait(), which returns once the predecessor
// has completed and its writes are visible, and only then touches global memory. Directly after its own wait it calls
// grid_launch_dependents(), so at most one successor runs ahead. Both calls are no-ops in a kernel launched the plain way,
// and a successor of a kernel that never signals simply starts when that kernel has finished.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// PDLLM_NO_PDL=1 launches every kernel the plain way (for A/B timing)
inline bool dependent_launch_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("PDLLM_NO_PDL");
    return !(v != nullptr && v[0] != '\0' && v[0] != '0');
  }();
  return on;
}

// Launch `kernel` on `stream`, overlapping its start with the tail of the kernel before it (see above). The kernel must call
// grid_dependency_wait() before its first access to global memory.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent_launch_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(std::forward<Args>(args))...);
}

inline int dtype_bytes(int dtype) { return dtype == PDLLM_F32 ? 4 : 2; }

// SM count of the CURRENT device (cached per device ordinal; benign race: every writer stores the same value)
inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

}  // namespace pdllm
