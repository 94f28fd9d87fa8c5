// NF4 blockwise codec: quantize / dequantize, on the device and on the host.
//
// Stands in for bitsandbytes.functional.quantize_4bit / dequantize_4bit as the
// reference calls them (experts4bit_qlora/_vendor/experts.py:408-426, 447-457):
// blocksize 64, fp32 absmax per block, no double quantization, two codes per
// byte with the first element in the high nibble. Quantization picks the
// nearest code of w * (1/absmax) with fp32 midpoint thresholds, a value exactly
// on a midpoint going to the lower code. Dequantization is
// dtype(code[q] * absmax) with a single round-to-nearest-even.
#include <cmath>
#include <cstring>

#include "common.cuh"

namespace e4b {

static const float h_nf4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

// One warp per 64-element block: two elements per lane.
template <typename T>
__global__ void nf4_quantize_kernel(const T* __restrict__ w, int64_t nblocks, uint8_t* __restrict__ packed,
                                    float* __restrict__ absmax) {
  __shared__ float thr[15];
  if (threadIdx.x < 15) thr[threadIdx.x] = __fmul_rn(__fadd_rn(c_nf4[threadIdx.x], c_nf4[threadIdx.x + 1]), 0.5f);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t b = warp; b < nblocks; b += nwarps) {
    float v0 = to_f32(w[b * 64 + 2 * lane]);
    float v1 = to_f32(w[b * 64 + 2 * lane + 1]);
    float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? __frcp_rn(m) : 0.f;
    const float s0 = __fmul_rn(v0, inv), s1 = __fmul_rn(v1, inv);
    int q0 = 0, q1 = 0;
#pragma unroll
    for (int i = 0; i < 15; ++i) {
      q0 += thr[i] < s0;
      q1 += thr[i] < s1;
    }
    packed[b * 32 + lane] = (uint8_t)((q0 << 4) | q1);
    if (lane == 0) absmax[b] = m;
  }
}

// Each thread decodes 4 packed bytes (8 elements) into one 16-byte store (two for fp32), so a
// warp reads 128 contiguous bytes and writes a contiguous run; the codebook is read from
// shared memory (lanes index it independently). out must be 16-byte aligned.
template <typename T> __device__ __forceinline__ uint32_t bits16(T v);
template <> __device__ __forceinline__ uint32_t bits16<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
template <> __device__ __forceinline__ uint32_t bits16<__half>(__half v) { return __half_as_ushort(v); }

template <typename T>
__global__ void __launch_bounds__(256) nf4_dequantize_kernel(const uint8_t* __restrict__ packed,
                                                             const float* __restrict__ absmax, int64_t ngroups,
                                                             T* __restrict__ out) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = c_nf4[threadIdx.x];
  __syncthreads();
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < ngroups; c += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t word = *reinterpret_cast<const uint32_t*>(packed + c * 4);
    const float a = absmax[c >> 3];  // 4 bytes = 8 elements = an eighth of a block
    float v[8];
#pragma unroll
    for (int bi = 0; bi < 4; ++bi) {
      const uint32_t byte = (word >> (8 * bi)) & 0xffu;
      v[2 * bi] = __fmul_rn(s_code[byte >> 4], a);
      v[2 * bi + 1] = __fmul_rn(s_code[byte & 15], a);
    }
    if constexpr (sizeof(T) == 4) {
      float4* o = reinterpret_cast<float4*>(out + c * 8);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w[j] = bits16<T>(from_f32<T>(v[2 * j])) | (bits16<T>(from_f32<T>(v[2 * j + 1])) << 16);
      *reinterpret_cast<uint4*>(out + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return (int)(g < 1 ? 1 : g);
}

// ---- host codec (same arithmetic, IEEE fp32) -----------------------------
static inline float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float host_load(const void* p, int dtype, int64_t i) {
  if (dtype == E4B_BF16) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p)[i]);
  if (dtype == E4B_F16) return (float)reinterpret_cast<const __half*>(p)[i];
  return reinterpret_cast<const float*>(p)[i];
}

}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_nf4_quantize(const void* w, int w_dtype, int64_t n, uint8_t* packed, float* absmax,
                                       void* stream) {
  if (n < 0 || n % 64 || (n && (!w || !packed || !absmax))) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(w_dtype)) return E4B_ERR_UNSUPPORTED;
  if (n == 0) return E4B_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t nb = n / 64;
  const int grid = grid_for(nb * 32, 256);
  if (w_dtype == E4B_BF16)
    nf4_quantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)w, nb, packed, absmax);
  else if (w_dtype == E4B_F16)
    nf4_quantize_kernel<__half><<<grid, 256, 0, s>>>((const __half*)w, nb, packed, absmax);
  else
    nf4_quantize_kernel<float><<<grid, 256, 0, s>>>((const float*)w, nb, packed, absmax);
  return launch_status();
}

extern "C" e4b_status e4b_nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n, void* out,
                                         int out_dtype, void* stream) {
  if (n < 0 || n % 64 || (n && (!packed || !absmax || !out))) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(out_dtype)) return E4B_ERR_UNSUPPORTED;
  if (n == 0) return E4B_OK;
  if (!aligned16(packed) || !aligned16(out)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t ngroups = n / 8;
  const int grid = grid_for(ngroups, 256);
  if (out_dtype == E4B_BF16)
    nf4_dequantize_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(packed, absmax, ngroups, (__nv_bfloat16*)out);
  else if (out_dtype == E4B_F16)
    nf4_dequantize_kernel<__half><<<grid, 256, 0, s>>>(packed, absmax, ngroups, (__half*)out);
  else
    nf4_dequantize_kernel<float><<<grid, 256, 0, s>>>(packed, absmax, ngroups, (float*)out);
  return launch_status();
}

extern "C" e4b_status e4b_nf4_quantize_host(const void* w, int w_dtype, int64_t n, uint8_t* packed,
                                            float* absmax) {
  if (n < 0 || n % 64 || (n && (!w || !packed || !absmax))) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(w_dtype)) return E4B_ERR_UNSUPPORTED;
  volatile float half = 0.5f;  // keep the threshold arithmetic in plain fp32
  float thr[15];
  for (int i = 0; i < 15; ++i) thr[i] = (h_nf4[i] + h_nf4[i + 1]) * half;
  for (int64_t b = 0; b < n / 64; ++b) {
    float v[64];
    float m = 0.f;
    for (int i = 0; i < 64; ++i) {
      v[i] = host_load(w, w_dtype, b * 64 + i);
      m = std::fmax(m, std::fabs(v[i]));
    }
    volatile float one = 1.0f;
    const float inv = m > 0.f ? one / m : 0.f;
    for (int i = 0; i < 64; i += 2) {
      volatile float s0 = v[i] * inv, s1 = v[i + 1] * inv;
      int q0 = 0, q1 = 0;
      for (int t = 0; t < 15; ++t) {
        q0 += thr[t] < s0;
        q1 += thr[t] < s1;
      }
      packed[b * 32 + i / 2] = (uint8_t)((q0 << 4) | q1);
    }
    absmax[b] = m;
  }
  return E4B_OK;
}

extern "C" e4b_status e4b_nf4_dequantize_host(const uint8_t* packed, const float* absmax, int64_t n, void* out,
                                              int out_dtype) {
  if (n < 0 || n % 64 || (n && (!packed || !absmax || !out))) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(out_dtype)) return E4B_ERR_UNSUPPORTED;
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t byte = packed[i >> 1];
    const int q = (i & 1) ? (byte & 15) : (byte >> 4);
    volatile float f = h_nf4[q] * absmax[i >> 6];
    if (out_dtype == E4B_BF16)
      reinterpret_cast<uint16_t*>(out)[i] = f32_to_bf16_rne(f);
    else if (out_dtype == E4B_F16)
      reinterpret_cast<__half*>(out)[i] = __float2half_rn(f);
    else
      reinterpret_cast<float*>(out)[i] = f;
  }
  return E4B_OK;
}
