// LoRA-A pre-pass (R5): xa[r, :] = scaling * (a_r . A[e]^T) for every sorted row r
// of expert e. This is the first factor of ExpertsLoRA._lora
// (experts4bit_qlora/lora.py:251-256); the second factor (. B[e]^T) and the add
// before the activation are fused into the grouped GEMM epilogue. Accumulation
// is fp32 whatever the adapter dtype.
#include "lora.cuh"

namespace e4b {

template <typename T>
__global__ void __launch_bounds__(256) lora_a_kernel(LoraAArgs g) {
  __shared__ float xs[kLoraRows][65];
  __shared__ float as[kLoraMaxRank][65];
  const int t = blockIdx.x;
  if (t >= g.tile_start[g.E]) return;
  int lo = 0, hi = g.E - 1;  // expert e with tile_start[e] <= t < tile_start[e+1]
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int e = lo;
  const int r0 = g.offsets[e] + (t - g.tile_start[e]) * kLoraRows;
  const int rend = g.offsets[e + 1];
  const int row = threadIdx.x >> 3, jg = threadIdx.x & 7;
  const T* A = reinterpret_cast<const T*>(g.a);
  float acc[kLoraMaxRank / 8];
#pragma unroll
  for (int i = 0; i < kLoraMaxRank / 8; ++i) acc[i] = 0.f;
  for (int k0 = 0; k0 < g.K; k0 += 64) {
    for (int i = threadIdx.x; i < kLoraRows * 64; i += blockDim.x) {
      const int rr = i >> 6, kk = i & 63;
      const int r = r0 + rr;
      float v = 0.f;
      if (r < rend) {
        const int64_t src = g.a_rows ? (int64_t)g.a_rows[r] : (int64_t)r;
        v = to_f32(A[src * g.K + k0 + kk]);
      }
      xs[rr][kk] = v;
    }
    for (int i = threadIdx.x; i < g.rank * 64; i += blockDim.x) {
      const int j = i >> 6, kk = i & 63;
      as[j][kk] = load_as_f32(g.loraA, g.lora_dtype, ((int64_t)e * g.rank + j) * g.K + k0 + kk);
    }
    __syncthreads();
    for (int kk = 0; kk < 64; ++kk) {
      const float xv = xs[row][kk];
#pragma unroll
      for (int i = 0; i < kLoraMaxRank / 8; ++i) {
        const int j = jg + 8 * i;
        if (j < g.rank) acc[i] = fmaf(xv, as[j][kk], acc[i]);
      }
    }
    __syncthreads();
  }
  const int r = r0 + row;
  if (r < rend) {
#pragma unroll
    for (int i = 0; i < kLoraMaxRank / 8; ++i) {
      const int j = jg + 8 * i;
      if (j < g.rank) g.xa[(int64_t)r * g.rank + j] = g.scaling * acc[i];
    }
  }
}

e4b_status launch_lora_a(const LoraAArgs& g, int act_dtype, cudaStream_t s) {
  if (g.max_tiles <= 0) return E4B_OK;
  if (act_dtype == E4B_BF16)
    lora_a_kernel<__nv_bfloat16><<<g.max_tiles, 256, 0, s>>>(g);
  else
    lora_a_kernel<__half><<<g.max_tiles, 256, 0, s>>>(g);
  return launch_status();
}

}  // namespace e4b
