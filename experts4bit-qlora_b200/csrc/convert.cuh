// Activation conversion for the fp16 tensor-core GEMV.
#pragma once
#include "common.cuh"

namespace e4b {

// Rows handled warp by warp: dst[r] = fp16(src[r] * 2^-s_r), scale[r] = 2^s_r,
// with the smallest s_r >= 0 keeping max|src[r]| * 2^-s_r <= 32768. Power-of-two
// scaling is exact, so a row inside the fp16 range (s_r = 0) converts exactly
// from bf16 (bf16's 8-bit significand fits fp16's 11 bits).
__device__ __forceinline__ void convert_rows_to_f16(const void* src, int src_dtype, __half* dst, float* scale,
                                                    int rows, int K, int first_warp, int num_warps) {
  const int lane = threadIdx.x & 31;
  for (int r = first_warp; r < rows; r += num_warps) {
    float m = 0.f;
    for (int k = lane; k < K; k += 32) m = fmaxf(m, fabsf(load_as_f32(src, src_dtype, (int64_t)r * K + k)));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int sh = 0;
    if (m > 32768.f) {
      int ex;
      frexpf(m / 32768.f, &ex);  // m / 32768 in [2^(ex-1), 2^ex)
      sh = ex;
    }
    const float inv = ldexpf(1.f, -sh);
    for (int k = lane; k < K; k += 32)
      dst[(int64_t)r * K + k] = __float2half_rn(load_as_f32(src, src_dtype, (int64_t)r * K + k) * inv);
    if (lane == 0) scale[r] = ldexpf(1.f, sh);
  }
}

struct ConvertArgs {
  const void* src;
  int src_dtype;
  __half* dst;
  float* scale;
  int rows, K;
};

}  // namespace e4b
