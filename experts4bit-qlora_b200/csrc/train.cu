// Element-wise kernels of the fused training path (train.py): the SwiGLU forward and
// backward over the expert-sorted projection rows, and the per-row gradients of the
// weighted combine. They replace chains of torch element-wise kernels over [R, 2I] and
// [R, H] tensors (casts, chunk, sigmoid, products, concatenation) with one pass each.
// Reference: the differentiable composition of engines/fast.py:453-552 (act(gate) * up
// between the projections, the top-k-weighted scatter of _scatter_combine, :260-278).
#include "common.cuh"

namespace e4b {
namespace {

// h = act(gate) * up as the reference computes it in the compute dtype: silu(gate) rounded
// to the dtype, times up, rounded again (without a gate: silu(x) rounded once).
template <typename T>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ proj, int64_t R, int I, int has_gate,
                                                         T* __restrict__ h) {
  const int64_t n = R * I;
  const int n1 = has_gate ? 2 * I : I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / I;
    const int c = (int)(i - r * I);
    const float g = to_f32(proj[r * n1 + c]);
    const float a = to_f32(from_f32<T>(g / (1.f + expf(-g))));
    h[i] = has_gate ? from_f32<T>(a * to_f32(proj[r * n1 + I + c])) : from_f32<T>(a);
  }
}

// dL/d(proj) from dL/dh (fp32): d gate = dh * up * s (1 + g (1 - s)), d up = dh * g s, with
// s = sigmoid(g); without a gate the first term with up = 1.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ proj, const float* __restrict__ dh,
                                                         int64_t R, int I, int has_gate, T* __restrict__ dproj) {
  const int64_t n = R * I;
  const int n1 = has_gate ? 2 * I : I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / I;
    const int c = (int)(i - r * I);
    const float g = to_f32(proj[r * n1 + c]);
    const float s = 1.f / (1.f + expf(-g));
    const float d = dh[i];
    const float dsilu = s * (1.f + g * (1.f - s));
    if (has_gate) {
      const float u = to_f32(proj[r * n1 + I + c]);
      dproj[r * n1 + c] = from_f32<T>(d * u * dsilu);
      dproj[r * n1 + I + c] = from_f32<T>(d * (g * s));
    } else {
      dproj[i] = from_f32<T>(d * dsilu);
    }
  }
}

// One block per expert-sorted row r (token t = rows[r]): dd[r] = grad[t] * w[r] in the compute
// dtype, dw[r] = sum_h grad[t, h] * down[r, h] in fp32 (block tree reduction, fixed order).
template <typename T>
__global__ void __launch_bounds__(256) row_grads_kernel(const float* __restrict__ grad, const int64_t* __restrict__ rows,
                                                        const float* __restrict__ w, const T* __restrict__ down, int H,
                                                        T* __restrict__ dd, float* __restrict__ dw) {
  __shared__ float red[256];
  const int64_t r = blockIdx.x;
  const int64_t t = rows[r];
  const float wr = w[r];
  const float* g = grad + t * H;
  const T* dn = down + r * H;
  float acc = 0.f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float gv = g[c];
    dd[r * H + c] = from_f32<T>(gv * wr);
    acc = fmaf(gv, to_f32(dn[c]), acc);
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) dw[r] = red[0];
}

inline int grid_for(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (int)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

}  // namespace
}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_swiglu_forward(const void* proj, int dtype, int64_t R, int I, int has_gate, void* h,
                                         void* stream) {
  if (R < 0 || I <= 0) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(dtype)) return E4B_ERR_UNSUPPORTED;
  if (R == 0) return E4B_OK;
  if (!proj || !h) return E4B_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = grid_for(R * I);
  if (dtype == E4B_BF16)
    swiglu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)proj, R, I, has_gate,
                                                          (__nv_bfloat16*)h);
  else
    swiglu_fwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)proj, R, I, has_gate, (__half*)h);
  return launch_status();
}

extern "C" e4b_status e4b_swiglu_backward(const void* proj, int dtype, const float* dh, int64_t R, int I, int has_gate,
                                          void* dproj, void* stream) {
  if (R < 0 || I <= 0) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(dtype)) return E4B_ERR_UNSUPPORTED;
  if (R == 0) return E4B_OK;
  if (!proj || !dh || !dproj) return E4B_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  const int grid = grid_for(R * I);
  if (dtype == E4B_BF16)
    swiglu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)proj, dh, R, I, has_gate,
                                                          (__nv_bfloat16*)dproj);
  else
    swiglu_bwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)proj, dh, R, I, has_gate, (__half*)dproj);
  return launch_status();
}

extern "C" e4b_status e4b_combine_row_grads(const float* grad, const int64_t* token_rows, const float* w_rows,
                                            const void* down, int dtype, int64_t R, int H, void* dd, float* dw,
                                            void* stream) {
  if (R < 0 || H <= 0) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(dtype)) return E4B_ERR_UNSUPPORTED;
  if (R == 0) return E4B_OK;
  if (!grad || !token_rows || !w_rows || !down || !dd || !dw) return E4B_ERR_INVALID_ARG;
  if (R > 0x7fffffff) return E4B_ERR_UNSUPPORTED;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == E4B_BF16)
    row_grads_kernel<__nv_bfloat16><<<(unsigned)R, 256, 0, s>>>(grad, token_rows, w_rows, (const __nv_bfloat16*)down,
                                                                H, (__nv_bfloat16*)dd, dw);
  else
    row_grads_kernel<__half><<<(unsigned)R, 256, 0, s>>>(grad, token_rows, w_rows, (const __half*)down, H,
                                                         (__half*)dd, dw);
  return launch_status();
}
