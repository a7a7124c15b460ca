// kb_common.cuh — shared helpers for the sm_100a operator kernels:
// status/error plumbing for the C ABI, streaming vector loads/stores, and
// deterministic warp/block reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>

#include <algorithm>

#include "../../include/kbb200.h"

namespace kb {

// ---------------------------------------------------------------------------
// error plumbing (defined in capi.cu)
// ---------------------------------------------------------------------------
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);          // cudaGetLastError -> status
int sm_count();                               // SMs of the current device
int max_smem_optin();                         // opt-in smem per block (bytes)

#define KB_REQUIRE(cond, status, ...)                  \
  do {                                                 \
    if (!(cond)) return ::kb::set_error((status), __VA_ARGS__); \
  } while (0)

#define KB_CUDA(call)                                                        \
  do {                                                                       \
    cudaError_t _e = (call);                                                 \
    if (_e != cudaSuccess)                                                   \
      return ::kb::set_error(KB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// memory access helpers
// ---------------------------------------------------------------------------
// Read-once data: streaming (evict-first) loads through the non-coherent path.
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ float ld_stream(const float* p) { return __ldcs(p); }
// Write-once data: streaming stores.
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float2* p, float2 v) { __stcs(p, v); }
__device__ __forceinline__ void st_stream(float* p, float v) { __stcs(p, v); }

// 256-bit accesses (sm_100): eight floats per instruction, 32-byte aligned.
struct f32x8 {
  float v[8];
};
__device__ __forceinline__ f32x8 ld_stream8(const float* p) {
  f32x8 r;
  asm volatile("ld.global.cs.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]),
                 "=f"(r.v[5]), "=f"(r.v[6]), "=f"(r.v[7])
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream8(float* p, const f32x8& r) {
  asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(r.v[0]),
               "f"(r.v[1]), "f"(r.v[2]), "f"(r.v[3]), "f"(r.v[4]), "f"(r.v[5]), "f"(r.v[6]),
               "f"(r.v[7])
               : "memory");
}

// ---------------------------------------------------------------------------
// reductions (fixed shuffle trees: results depend only on the launch shape)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; every thread gets the result.  `red` holds >= 32 values.
// Ends with the shared buffer free for reuse after a following barrier.
template <int NT, typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  static_assert(NT % 32 == 0 && NT <= 1024, "block size");
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (NW == 1) return v;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T r = (lane < NW) ? red[lane] : T(0);
  r = warp_sum(r);
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (NW == 1) return v;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = (lane < NW) ? red[lane] : -INFINITY;
  r = warp_max(r);
  __syncthreads();
  return r;
}

}  // namespace kb
