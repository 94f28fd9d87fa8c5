// Activation conversion for the fp16 tensor-core GEMV.
#pragma once
#include "common.cuh"

namespace e4b {

// Rows handled warp by warp: dst[r] = fp16(src[r] * 2^-s_r), scale[r] = 2^s_r,
// with the smallest s_r >= 0 keeping max|src[r]| * 2^-s_r <= 32768. Power-of-two
// scaling is exact, so a row inside the fp16 range (s_r = 0) converts exactly
// from bf16 (bf16's 8-bit significand fits fp16's 11 bits).
__device__ __forceinline__ void load8(const void* src, int dtype, int64_t i, float (&v)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(src) + i * 2);
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (dtype == E4B_BF16) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void expand8(uint4 r, int dtype, float (&v)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (dtype == E4B_BF16) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// Rows of a 16-bit (bf16/fp16) source, K % 8 == 0, one warp per row. Up to 8 16-byte vectors per
// lane stay in registers as loaded (16-bit, 32 registers) so the row is read once with all loads
// in flight and the kernel keeps a high occupancy (longer rows take a second, cached read); they
// are expanded to fp32 twice, for the row maximum and for the scaled store.
__device__ __forceinline__ void convert_rows_to_f16(const void* src, int src_dtype, __half* dst, float* scale,
                                                    int rows, int K, int first_warp, int num_warps) {
  const int lane = threadIdx.x & 31;
  const int nv = K / 8;
  for (int r = first_warp; r < rows; r += num_warps) {
    const int64_t base = (int64_t)r * K;
    uint4 raw[8];
    float m = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = lane + 32 * u;
      raw[u] = c < nv ? *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(src) + (base + c * 8) * 2)
                      : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float v[8];
      expand8(raw[u], src_dtype, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
    }
    for (int c = lane + 256; c < nv; c += 32) {
      float t[8];
      load8(src, src_dtype, base + c * 8, t);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(t[j]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int sh = 0;
    if (m > 32768.f) {
      int ex;
      frexpf(m / 32768.f, &ex);  // m / 32768 in [2^(ex-1), 2^ex)
      sh = ex;
    }
    const float inv = ldexpf(1.f, -sh);
    auto put = [&](int c, const float (&t)[8]) {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) ow[j] = pack2<__half>(t[2 * j] * inv, t[2 * j + 1] * inv);
      *reinterpret_cast<uint4*>(dst + base + c * 8) = o;
    };
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (lane + 32 * u < nv) {
        float v[8];
        expand8(raw[u], src_dtype, v);
        put(lane + 32 * u, v);
      }
    for (int c = lane + 256; c < nv; c += 32) {
      float t[8];
      load8(src, src_dtype, base + c * 8, t);
      put(c, t);
    }
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
