// LoRA-A pre-pass (R5): xa[r, :] = scaling * (a_r . A[e]^T) for every sorted row r
// of expert e -- the first factor of ExpertsLoRA._lora (experts4bit_qlora/lora.py:
// 251-256); the second factor (. B[e]^T) and the add before the activation are
// fused into the grouped GEMM epilogues.
//
// A CTA takes 64 rows of one expert; each of its 4 warps computes 16 rows x all
// ranks with mma.sync m16n8k16 (fp16 operands, fp32 accumulation), the 64-wide K
// chunks of the rows and of A[e] staged in padded shared memory.
#include "lora.cuh"

namespace e4b {

namespace {
// K chunk per shared-memory round: 256 for ranks <= 16 (fewer barriers and more loads in flight),
// 64 above (the A tile grows with the rank); rows padded by 8 halves keep fragment reads
// conflict free.
template <int NR> struct LoraChunk { static constexpr int kc = NR <= 2 ? 256 : 64; };

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
}  // namespace

template <int NR>  // n8 tiles of ranks: rank <= 8 * NR
__global__ void __launch_bounds__(128) lora_a_kernel(LoraAArgs g) {
  constexpr int kKc = LoraChunk<NR>::kc;
  constexpr int kPitch = kKc + 8;
  __shared__ __align__(16) __half xs[kLoraRows][kPitch];
  __shared__ __align__(16) __half as[8 * NR][kPitch];
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, q = lane & 3;
  float acc[NR][4];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
  for (int k0 = 0; k0 < g.K; k0 += kKc) {
    for (int i = threadIdx.x; i < kLoraRows * (kKc / 8); i += blockDim.x) {
      const int rr = i / (kKc / 8), v = i % (kKc / 8);
      const int r = r0 + rr;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (r < rend && k0 + v * 8 < g.K) {  // zero past K: a chunk may overrun a K that is a multiple of 64
        const int64_t src = g.a_rows ? (int64_t)g.a_rows[r] : (int64_t)r;
        val = *reinterpret_cast<const uint4*>(g.a + src * g.K + k0 + v * 8);
      }
      *reinterpret_cast<uint4*>(&xs[rr][v * 8]) = val;
    }
    for (int i = threadIdx.x; i < 8 * NR * kKc; i += blockDim.x) {
      const int j = i / kKc, kk = i % kKc;
      const float v = (j < g.rank && k0 + kk < g.K)
                          ? load_as_f32(g.loraA, g.lora_dtype, ((int64_t)e * g.rank + j) * g.K + k0 + kk)
                          : 0.f;
      as[j][kk] = __float2half_rn(v);
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < kKc; ks += 16) {
      const int rw = warp * 16 + gq;
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&xs[rw][ks + 2 * q]);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(&xs[rw + 8][ks + 2 * q]);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&xs[rw][ks + 2 * q + 8]);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(&xs[rw + 8][ks + 2 * q + 8]);
#pragma unroll
      for (int n = 0; n < NR; ++n) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&as[n * 8 + gq][ks + 2 * q]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&as[n * 8 + gq][ks + 2 * q + 8]);
        mma_f16(acc[n], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + warp * 16 + gq + 8 * h;
    if (r >= rend) continue;
    if (g.xa16) {  // fp16, no activation scale: the GEMM's epilogue applies it to the whole accumulator
#pragma unroll
      for (int n = 0; n < NR; ++n) {
        const int j = n * 8 + 2 * q;
        if (j < 16)
          *reinterpret_cast<__half2*>(g.xa16 + (int64_t)r * 64 + j) =
              __floats2half2_rn(j < g.rank ? g.scaling * acc[n][2 * h] : 0.f,
                                j + 1 < g.rank ? g.scaling * acc[n][2 * h + 1] : 0.f);
      }
      if (NR == 1) {  // ranks <= 8: the second 8 of the 16 columns are zero
        *reinterpret_cast<__half2*>(g.xa16 + (int64_t)r * 64 + 8 + 2 * q) = __floats2half2_rn(0.f, 0.f);
      }
      continue;
    }
    float sc = g.scaling;
    if (g.a_scale) sc *= g.a_scale[g.a_rows ? g.a_rows[r] : r];
#pragma unroll
    for (int n = 0; n < NR; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int j = n * 8 + 2 * q + c;
        if (j < g.rank) g.xa[(int64_t)r * g.rank + j] = sc * acc[n][2 * h + c];
      }
  }
}

e4b_status launch_lora_a(const LoraAArgs& g, cudaStream_t s) {
  if (g.max_tiles <= 0) return E4B_OK;
  if (g.K % 64) return E4B_ERR_UNSUPPORTED;
  const int nr = (g.rank + 7) / 8;
  if (nr <= 1)
    lora_a_kernel<1><<<g.max_tiles, 128, 0, s>>>(g);
  else if (nr <= 2)
    lora_a_kernel<2><<<g.max_tiles, 128, 0, s>>>(g);
  else if (nr <= 4)
    lora_a_kernel<4><<<g.max_tiles, 128, 0, s>>>(g);
  else
    lora_a_kernel<8><<<g.max_tiles, 128, 0, s>>>(g);
  return launch_status();
}

}  // namespace e4b
