// Shared device/host helpers for the GDN-2 sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gdn2.h"

namespace gdn2 {

// Device-side strided view: element pointer + element strides of dims 0..2.
struct DView {
  const void* p;
  int64_t s0, s1, s2;
};

__host__ inline DView make_dview(const gdn2_view& v) { return DView{v.data, v.stride0, v.stride1, v.stride2}; }

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Element (i0, i1, i2, i3) of a view, read as f32.
template <typename T>
__device__ __forceinline__ float vload(const DView& v, int64_t i0, int64_t i1, int64_t i2, int64_t i3) {
  const T* p = static_cast<const T*>(v.p);
  return to_f32<T>(p[i0 * v.s0 + i1 * v.s1 + i2 * v.s2 + i3]);
}

template <typename T>
__device__ __forceinline__ void vstore(const DView& v, int64_t i0, int64_t i1, int64_t i2, int64_t i3, float x) {
  T* p = static_cast<T*>(const_cast<void*>(v.p));
  p[i0 * v.s0 + i1 * v.s1 + i2 * v.s2 + i3] = from_f32<T>(x);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Block-wide sum for blockDim.x == NT (multiple of 32).  `red` holds >= 32 floats.
template <int NT>
__device__ __forceinline__ float block_sum(float x, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = (lane < NT / 32) ? red[lane] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[0] = s;
  }
  __syncthreads();
  s = red[0];
  __syncthreads();
  return s;
}

}  // namespace gdn2

// ---- host-side error reporting (api.cu) ----
namespace gdn2 {
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* where);
// SMs of the current device less those reserved by gdn2_set_reserved_sms (148 on a B200 if the query fails)
int usable_sms();
}  // namespace gdn2
