// Shared device helpers for libe4b (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "e4b.h"

namespace e4b {

// The 16 NF4 values (QLoRA, arXiv:2305.14314, Appendix E); each an exact float32.
static __constant__ float c_nf4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

// Workspace header: the device error word (first 4 bytes, sticky: set by the first error, cleared
// only by e4b_read_device_error), a few words some entry points use, and at kFlowSyncOffset the
// counter block of the flow decode kernel (zero when idle). Every layout starts after it.
constexpr size_t kErrBytes = 1024;
constexpr size_t kFlowSyncOffset = 512;
constexpr int kFlowDiagWord = 16;  // int words 16..20: the flow kernel's first timed-out wait

__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Pack two floats into one 32-bit register of T2 (low half = first).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case E4B_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case E4B_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

// Store with the fp16 range guarded: values beyond +-65504 saturate and raise
// E4B_ERR_RANGE (a bf16 store never saturates).
template <typename T> __device__ __forceinline__ T store_cast(float v, int* err);
template <> __device__ __forceinline__ __nv_bfloat16 store_cast<__nv_bfloat16>(float v, int*) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half store_cast<__half>(float v, int* err) {
  if (fabsf(v) > 65504.f) {
    raise_error(err, E4B_ERR_RANGE);
    v = copysignf(65504.f, v);
  }
  return __float2half_rn(v);
}

// Stack index of a routed expert id. Without a map the id indexes the [E, ...] stacks directly;
// with one (a resident sub-stack), ids lie in [0, routed) and map[id] is the expert's index in the
// stacks (-1: not resident). Ids that land outside [0, E) are clamped for memory safety and
// reported as E4B_ERR_EXPERT_INDEX when `report`.
__device__ __forceinline__ int stack_expert(int64_t raw, const int32_t* map, int routed, int E, int* err,
                                            bool report) {
  if (map) {
    if (raw < 0 || raw >= routed) {
      if (report) raise_error(err, E4B_ERR_EXPERT_INDEX);
      return raw < 0 ? 0 : E - 1;
    }
    raw = map[raw];
  }
  if (raw < 0 || raw >= E) {
    if (report) raise_error(err, E4B_ERR_EXPERT_INDEX);
    return raw < 0 ? 0 : E - 1;
  }
  return (int)raw;
}

__device__ __forceinline__ float silu_f32(float g) { return g / (1.0f + __expf(-g)); }

// Streaming 64-bit global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline e4b_status launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? E4B_OK : E4B_ERR_CUDA;
}

inline bool is_act_dtype(int d) { return d == E4B_BF16 || d == E4B_F16; }
inline bool is_any_dtype(int d) { return d == E4B_BF16 || d == E4B_F16 || d == E4B_F32; }

}  // namespace e4b
