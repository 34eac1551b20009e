// common.cuh -- shared device helpers for the sm_100a sparse front-end kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/bjf.h"

namespace bjf {

// Element conversion -------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Eight consecutive elements through 16-byte vector accesses.  The pointer
// must be 16-byte aligned (32-byte for float).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename H>
__device__ __forceinline__ void load8_16bit(const H* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const H* h = reinterpret_cast<const H*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = to_f32<H>(h[i]);
}
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  load8_16bit<__half>(p, v);
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  load8_16bit<__nv_bfloat16>(p, v);
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
template <typename H>
__device__ __forceinline__ void store8_16bit(H* p, const float (&v)[8]) {
  uint4 u;
  H* h = reinterpret_cast<H*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = from_f32<H>(v[i]);
  *reinterpret_cast<uint4*>(p) = u;
}
template <>
__device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  store8_16bit<__half>(p, v);
}
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  store8_16bit<__nv_bfloat16>(p, v);
}

// Streaming 16-byte load that does not allocate in L1 (read-once data).
// Streaming 16-byte load: no L1 allocation, and evict-first in L2 so a pass over hundreds of
// MB leaves the lines other kernels reuse (the GEMM's gathered rows and weights) in place.
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  uint64_t policy;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(policy));
  return r;
}

__host__ __device__ constexpr int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  A kernel launched with pdl = true may start while the
// kernel before it in the stream is still running; pdl_wait() blocks until that kernel has
// completed and its writes are visible (it returns at once for an ordinary launch).
// pdl_trigger() lets the next kernel of the stream, if it was launched with pdl = true,
// start before this one completes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches `kernel`, optionally as a programmatic dependent of the previous kernel.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, Args&&... args) {
  if (!pdl) {
    kernel<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline size_t dtype_size(int32_t dt) {
  switch (dt) {
    case BJF_DTYPE_F32: return 4;
    case BJF_DTYPE_F16: return 2;
    case BJF_DTYPE_BF16: return 2;
    case BJF_DTYPE_I32: return 4;
    default: return 0;
  }
}

// Dispatch a functor over the three float element types.
template <typename F>
inline bool dispatch_float(int32_t dt, F&& f) {
  switch (dt) {
    case BJF_DTYPE_F32: f(float{}); return true;
    case BJF_DTYPE_F16: f(__half{}); return true;
    case BJF_DTYPE_BF16: f(__nv_bfloat16{}); return true;
    default: return false;
  }
}

}  // namespace bjf
