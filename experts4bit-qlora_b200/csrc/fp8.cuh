// Block-scaled FP8 (e4m3) weight decode shared by the FP8 kernels.
#pragma once
#include <cuda_fp8.h>

#include "common.cuh"

namespace e4b {

constexpr int kFp8Block = 128;  // scale tile edge (formats/fp8_blocks.py BLOCK)

// Two e4m3 bytes (low byte first) -> fp16x2 bits, exactly.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two_bytes & 0xffffu), __NV_E4M3);
  return (uint32_t)hr.x | ((uint32_t)hr.y << 16);
}

// Two e4m3 bytes (low byte first) -> fp32 values, exactly (e4m3 fits fp16).
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t two_bytes) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two_bytes & 0xffffu), __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&hr));
}

// fp16x2 of (fp32(w) * r) for two e4m3 bytes (r a ratio of tile scales, <= 1).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2_scaled(uint32_t two_bytes, float r) {
  const float2 f = e4m3x2_to_f32x2(two_bytes);
  return pack2<__half>(f.x * r, f.y * r);
}

}  // namespace e4b
