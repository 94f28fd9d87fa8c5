// MXFP4 (OCP Microscaling FP4) expert weights: dequantization, device and host.
//
// The storage of formats/mxfp4.py:1-105 (gpt-oss and DeepSeek-V3-lineage
// checkpoints): blocks uint8 [P, rows, G, B], two e2m1 codes per byte with the
// LOW nibble first; scales uint8 [P, rows, G], one e8m0 exponent (bias 127) per
// block of 2B values. The value of code c under scale s is
// fp32(E2M1[c]) * 2^(s-127) -- exact in fp32, the subnormal 2^-127 included --
// rounded once to the output dtype, and the result is laid out [P, G*2B, rows]
// (the trailing (rows, K) pair transposed), as the reference returns it.
#include <cstring>

#include "common.cuh"

namespace e4b {

namespace {

__constant__ float c_e2m1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                 -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
const float h_e2m1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                          -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// 2^(s-127) as fp32 bits: s << 23 for s >= 1 (s = 255 gives +inf, as 2.0**128 does in fp32);
// s = 0 is the subnormal 2^-127 (mantissa bit 22).
__host__ __device__ __forceinline__ uint32_t e8m0_bits(uint32_t s) { return s ? s << 23 : 0x00400000u; }

__host__ __device__ __forceinline__ float e8m0_value(uint32_t s) {
  const uint32_t b = e8m0_bits(s);
  float f;
  memcpy(&f, &b, 4);
  return f;
}

// code * 2^(s-127) exactly as ldexp (the reference's torch.ldexp) gives it: one rounding of the
// exact product. For s <= 254 the factor is a float and one multiply is exact or rounds once; for
// s = 255 the factor 2^128 is not, so the product is formed as (code * 2^64) * 2^64: 0.5 * 2^128
// stays finite, codes >= 1 overflow to inf, zero stays a signed zero (no 0 * inf = NaN).
__device__ __forceinline__ float e8m0_scale_dev(float c, uint32_t s) {
  if (s == 255u) return __fmul_rn(__fmul_rn(c, 18446744073709551616.0f), 18446744073709551616.0f);
  return __fmul_rn(c, e8m0_value(s));
}
inline float e8m0_scale_host(float c, uint32_t s) {
  volatile float v;
  if (s == 255u) {
    v = c * 18446744073709551616.0f;
    v = v * 18446744073709551616.0f;
  } else {
    v = c * e8m0_value(s);
  }
  return v;
}

// One thread per output element (p, k, r), r fastest: the stores are coalesced; each
// warp reads its rows' bytes of one 2-element column pair (served by L1/L2).
template <typename T>
__global__ void __launch_bounds__(256) mxfp4_dequant_kernel(const uint8_t* __restrict__ blocks,
                                                            const uint8_t* __restrict__ scales, int64_t P,
                                                            int64_t rows, int64_t G, int64_t B,
                                                            T* __restrict__ out) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = c_e2m1[threadIdx.x];
  __syncthreads();
  const int64_t K = G * 2 * B, n = P * K * rows;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i % rows, pk = i / rows, k = pk % K, p = pk / K;
    const int64_t row = p * rows + r;
    const uint32_t byte = blocks[row * G * B + (k >> 1)];
    const uint32_t code = (k & 1) ? byte >> 4 : byte & 15u;
    const float v = e8m0_scale_dev(s_code[code], scales[row * G + k / (2 * B)]);
    out[i] = from_f32<T>(v);
  }
}

bool mxfp4_args_ok(const uint8_t* blocks, const uint8_t* scales, int64_t P, int64_t rows, int64_t G, int64_t B,
                   const void* out) {
  if (P < 0 || rows < 0 || G < 0 || B <= 0) return false;
  if (P * rows * G * B > ((int64_t)1 << 40)) return false;
  if (P * rows * G > 0 && (!blocks || !scales || !out)) return false;
  return true;
}

template <typename T> T host_cast(float v);
template <> float host_cast<float>(float v) { return v; }
template <> __nv_bfloat16 host_cast<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __half host_cast<__half>(float v) { return __float2half_rn(v); }

template <typename T>
void mxfp4_dequant_host(const uint8_t* blocks, const uint8_t* scales, int64_t P, int64_t rows, int64_t G, int64_t B,
                        T* out) {
  const int64_t K = G * 2 * B;
  for (int64_t p = 0; p < P; ++p)
    for (int64_t r = 0; r < rows; ++r) {
      const int64_t row = p * rows + r;
      for (int64_t k = 0; k < K; ++k) {
        const uint32_t byte = blocks[row * G * B + (k >> 1)];
        const uint32_t code = (k & 1) ? byte >> 4 : byte & 15u;
        const float v = e8m0_scale_host(h_e2m1[code], scales[row * G + k / (2 * B)]);
        out[(p * K + k) * rows + r] = host_cast<T>(v);
      }
    }
}

}  // namespace

}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_mxfp4_dequantize(const uint8_t* blocks, const uint8_t* scales, int64_t P, int64_t rows,
                                          int64_t G, int64_t B, void* out, int out_dtype, void* stream) {
  if (!mxfp4_args_ok(blocks, scales, P, rows, G, B, out)) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(out_dtype)) return E4B_ERR_UNSUPPORTED;
  const int64_t n = P * rows * G * 2 * B;
  if (n == 0) return E4B_OK;
  cudaStream_t s = (cudaStream_t)stream;
  int64_t g = (n + 255) / 256;
  if (g > 148 * 16) g = 148 * 16;
  if (out_dtype == E4B_BF16)
    mxfp4_dequant_kernel<__nv_bfloat16><<<(int)g, 256, 0, s>>>(blocks, scales, P, rows, G, B,
                                                               static_cast<__nv_bfloat16*>(out));
  else if (out_dtype == E4B_F16)
    mxfp4_dequant_kernel<__half><<<(int)g, 256, 0, s>>>(blocks, scales, P, rows, G, B, static_cast<__half*>(out));
  else
    mxfp4_dequant_kernel<float><<<(int)g, 256, 0, s>>>(blocks, scales, P, rows, G, B, static_cast<float*>(out));
  return launch_status();
}

extern "C" e4b_status e4b_mxfp4_dequantize_host(const uint8_t* blocks_host, const uint8_t* scales_host, int64_t P,
                                               int64_t rows, int64_t G, int64_t B, void* out_host, int out_dtype) {
  if (!mxfp4_args_ok(blocks_host, scales_host, P, rows, G, B, out_host)) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(out_dtype)) return E4B_ERR_UNSUPPORTED;
  if (out_dtype == E4B_BF16)
    mxfp4_dequant_host(blocks_host, scales_host, P, rows, G, B, static_cast<__nv_bfloat16*>(out_host));
  else if (out_dtype == E4B_F16)
    mxfp4_dequant_host(blocks_host, scales_host, P, rows, G, B, static_cast<__half*>(out_host));
  else
    mxfp4_dequant_host(blocks_host, scales_host, P, rows, G, B, static_cast<float*>(out_host));
  return E4B_OK;
}
