// Weighted, deterministic un-permute (R7): replaces engines/fast.py:158-160 and
// _scatter_combine (:260-278). out[t] = sum over s = 0..k-1, in slot order, of
// fp32(rows[inv[t*k+s]]) * fp32(w[t,s]) (w = NULL: weight 1, the plain slot sum the
// training backward needs for dL/dx); no atomics, so repeated calls are bit-identical.
#include "common.cuh"

namespace e4b {

constexpr int kMaxK = 32;

template <typename TR, typename TO>
__global__ void __launch_bounds__(256) combine_kernel(const TR* __restrict__ rows, const int32_t* __restrict__ inv,
                                                      const void* __restrict__ w, int w_dtype, int k, int H,
                                                      TO* __restrict__ out) {
  // the token's k (row, weight) pairs first, then every row load at once: two
  // dependent memory round trips per token instead of one per slot
  __shared__ int64_t s_row[kMaxK];
  __shared__ float s_w[kMaxK];
  const int t = blockIdx.x;
  if (threadIdx.x < k) {
    s_row[threadIdx.x] = (int64_t)inv[(int64_t)t * k + threadIdx.x] * H;
    s_w[threadIdx.x] = w ? load_as_f32(w, w_dtype, (int64_t)t * k + threadIdx.x) : 1.f;
  }
  __syncthreads();
  for (int h = threadIdx.x * 8; h < H; h += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    constexpr int kVec = sizeof(TR) == 4 ? 2 : 1;  // 16-byte vectors per 8 elements
    for (int s0 = 0; s0 < k; s0 += 8) {
      uint4 v[8][kVec];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < k)
#pragma unroll
          for (int q = 0; q < kVec; ++q) v[u][q] = reinterpret_cast<const uint4*>(rows + s_row[s0 + u] + h)[q];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + u >= k) break;
        const TR* vv = reinterpret_cast<const TR*>(&v[u][0]);
        const float ws = s_w[s0 + u];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(to_f32(vv[i]), ws, acc[i]);  // slot order
      }
    }
    TO o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = from_f32<TO>(acc[i]);
    if (sizeof(TO) == 2) {
      *reinterpret_cast<uint4*>(out + (int64_t)t * H + h) = *reinterpret_cast<uint4*>(o);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[(int64_t)t * H + h + i] = o[i];
    }
  }
}

template <typename TR>
static void launch_rows(const void* rows, const int32_t* inv, const void* w, int w_dtype, int T, int k, int H,
                        void* out, int out_dtype, cudaStream_t s) {
  if (out_dtype == E4B_BF16)
    combine_kernel<TR, __nv_bfloat16><<<T, 256, 0, s>>>((const TR*)rows, inv, w, w_dtype, k, H, (__nv_bfloat16*)out);
  else if (out_dtype == E4B_F16)
    combine_kernel<TR, __half><<<T, 256, 0, s>>>((const TR*)rows, inv, w, w_dtype, k, H, (__half*)out);
  else
    combine_kernel<TR, float><<<T, 256, 0, s>>>((const TR*)rows, inv, w, w_dtype, k, H, (float*)out);
}

}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_combine(const void* rows, int rows_dtype, const int32_t* inv, const void* w, int w_dtype,
                                  int T, int k, int H, void* out, int out_dtype, void* stream) {
  if (T < 0 || k <= 0 || k > kMaxK || H <= 0) return E4B_ERR_INVALID_ARG;
  if (!(is_act_dtype(rows_dtype) || rows_dtype == E4B_F32) || (w && !is_any_dtype(w_dtype)) ||
      !is_any_dtype(out_dtype) || H % 8)
    return E4B_ERR_UNSUPPORTED;
  if (T == 0) return E4B_OK;
  if (!rows || !inv || !out) return E4B_ERR_INVALID_ARG;
  if (!aligned16(rows) || !aligned16(out)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  if (rows_dtype == E4B_BF16)
    launch_rows<__nv_bfloat16>(rows, inv, w, w_dtype, T, k, H, out, out_dtype, s);
  else if (rows_dtype == E4B_F32)
    launch_rows<float>(rows, inv, w, w_dtype, T, k, H, out, out_dtype, s);
  else
    launch_rows<__half>(rows, inv, w, w_dtype, T, k, H, out, out_dtype, s);
  return launch_status();
}
