// Grouped NF4 GEMV for the decode regime (few tokens per expert).
//
// Replaces grouped-nf4-gemm's gemm_4bit_grouped at decode shapes
// (experts4bit_qlora/engines/fast.py:137-156) with the gate_up epilogue
// (lora._epilogue, lora.py:102-128) and the LoRA delta (lora.py:251-256) fused.
//
// The weights are HBM-streamed exactly once. Each warp owns 16 weight rows (an
// m16 tensor-core tile; for SwiGLU 8 gate rows + the 8 matching up rows, so one
// lane ends up holding gate and up of the same output feature) and a 1/8 slice
// of K. Per 64-element quantization block, a lane reads 8 packed bytes of each
// of its two rows (64-bit streaming loads), turns each byte into a bf16/fp16
// pair with ONE shared-memory lookup in a 256-entry pair table replicated per
// lane (entry e of lane l at byte (e << 8) | (l << 2): the address is a single
// byte-permute and no two lanes ever hit the same bank), and feeds the pairs
// straight into register A fragments of mma.sync m16n8k16 whose B operand is
// the activations (<= 8 tokens per n8 tile). The block's partial sum is scaled
// by its fp32 absmax in fp32, so the code -> weight scaling never rounds.
// The MMA runs in fp16: the 16 codes carry 11 significant bits there (bf16
// would round them by up to 2^-8, a systematic per-code error that costs
// ~1.4e-3 of relative output error), and the activations arrive as fp16 with a
// per-row power-of-two scale (convert.cu) that keeps them in range exactly.
// The K dimension is permuted consistently on A and B (both sides read the
// same physical elements), which lets each lane's bytes stay contiguous.
#include "gemv.cuh"

namespace e4b {

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kLutBytes = 256 * 256;       // 256 entries x 256-byte stride (lanes in the low 128)
constexpr int kUnroll = 4;                 // quantization blocks in flight per warp

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct MmaOp<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

// Pair table: entry `byte` = {code[byte >> 4] (low half, first element), code[byte & 15]}.
template <typename T>
__device__ __forceinline__ void build_pair_lut(uint32_t* lut) {
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int e = i >> 5, l = i & 31;
    lut[e * 64 + l] = pack2<T>(c_nf4[e >> 4], c_nf4[e & 15]);
  }
}

template <int POS>
__device__ __forceinline__ uint32_t lut_pair(const char* lut, uint32_t word, uint32_t lane4) {
  // address = (byte POS of word) << 8 | lane * 4
  const uint32_t addr = __byte_perm(word, lane4, 0x5504u | (POS << 4));
  return *reinterpret_cast<const uint32_t*>(lut + addr);
}

__device__ __forceinline__ float lora_delta(const GemvArgs& g, int e, int row, int64_t srow) {
  float d = 0.f;
  const float* xa = g.lora_xa + srow * g.rank;
  const int64_t bbase = ((int64_t)e * g.N + row) * g.rank;
  for (int j = 0; j < g.rank; ++j) d = fmaf(xa[j], load_as_f32(g.lora_B, g.lora_dtype, bbase + j), d);
  return d;
}

template <typename OutT, int NT>
__global__ void __launch_bounds__(kGemvThreads, 3) nf4_gemv_kernel(GemvArgs g) {
  using T = __half;
  extern __shared__ __align__(16) uint32_t smem[];
  const char* lut = reinterpret_cast<const char*>(smem);
  float* red = reinterpret_cast<float*>(reinterpret_cast<char*>(smem) + kLutBytes);  // [warps][NT][4][32]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  const int nblk = g.K >> 6;
  const int64_t row_bytes = g.K >> 1;
  const int64_t am_row = g.K >> 6;
  const T* A = reinterpret_cast<const T*>(g.a);

  build_pair_lut<T>(smem);
  __syncthreads();

  const int num_active = *g.num_active;
  for (int task = blockIdx.x; task < g.max_tasks; task += gridDim.x) {
    const int j = task / g.tiles_per_expert;
    const int tile = task - j * g.tiles_per_expert;
    if (j >= num_active) break;  // tasks are ordered by active-expert slot
    const int e = g.active[j];
    const int row0 = g.offsets[e];
    const int M = g.offsets[e + 1] - row0;
    int rA, rB;
    if (g.epilogue == E4B_EPI_SWIGLU) {
      rA = tile * 8 + gq;
      rB = (g.N >> 1) + tile * 8 + gq;
    } else {
      rA = tile * 16 + gq;
      rB = rA + 8;
    }
    const uint8_t* pk = g.packed + (int64_t)e * g.N * row_bytes;
    const float* am = g.absmax + (int64_t)e * g.N * am_row;
    const uint8_t* pa = pk + (int64_t)rA * row_bytes + q * 8;
    const uint8_t* pb = pk + (int64_t)rB * row_bytes + q * 8;
    const float* ama = am + (int64_t)rA * am_row;
    const float* amb = am + (int64_t)rB * am_row;

    for (int m0 = 0; m0 < M; m0 += NT * 8) {
      const T* xrow[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = m0 + nt * 8 + gq;
        if (m < M) {
          const int64_t src = g.a_rows ? (int64_t)g.a_rows[row0 + m] : (int64_t)(row0 + m);
          xrow[nt] = A + src * g.K + q * 16;
        } else {
          xrow[nt] = nullptr;
        }
      }
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;

      for (int b0 = warp; b0 < nblk; b0 += kGemvWarps * kUnroll) {
        uint2 wa[kUnroll], wb[kUnroll];
        float sa[kUnroll], sb[kUnroll];
        uint4 xf[kUnroll][NT][2];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int b = b0 + u * kGemvWarps;
          if (b < nblk) {
            wa[u] = ldg_stream_u2(pa + b * 32);
            wb[u] = ldg_stream_u2(pb + b * 32);
            sa[u] = __ldg(ama + b);
            sb[u] = __ldg(amb + b);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (xrow[nt]) {
                xf[u][nt][0] = ldg_u4(xrow[nt] + b * 64);
                xf[u][nt][1] = ldg_u4(xrow[nt] + b * 64 + 8);
              } else {
                xf[u][nt][0] = make_uint4(0, 0, 0, 0);
                xf[u][nt][1] = make_uint4(0, 0, 0, 0);
              }
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int b = b0 + u * kGemvWarps;
          if (b < nblk) {
            float p[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int r = 0; r < 4; ++r) p[nt][r] = 0.f;
            // MMA jj uses bytes 2jj (cols 2q,2q+1) and 2jj+1 (cols 2q+8,2q+9)
            {
              const uint32_t a0 = lut_pair<0>(lut, wa[u].x, lane4), a2 = lut_pair<1>(lut, wa[u].x, lane4);
              const uint32_t a1 = lut_pair<0>(lut, wb[u].x, lane4), a3 = lut_pair<1>(lut, wb[u].x, lane4);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(p[nt], a0, a1, a2, a3, xf[u][nt][0].x, xf[u][nt][0].y);
            }
            {
              const uint32_t a0 = lut_pair<2>(lut, wa[u].x, lane4), a2 = lut_pair<3>(lut, wa[u].x, lane4);
              const uint32_t a1 = lut_pair<2>(lut, wb[u].x, lane4), a3 = lut_pair<3>(lut, wb[u].x, lane4);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(p[nt], a0, a1, a2, a3, xf[u][nt][0].z, xf[u][nt][0].w);
            }
            {
              const uint32_t a0 = lut_pair<0>(lut, wa[u].y, lane4), a2 = lut_pair<1>(lut, wa[u].y, lane4);
              const uint32_t a1 = lut_pair<0>(lut, wb[u].y, lane4), a3 = lut_pair<1>(lut, wb[u].y, lane4);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(p[nt], a0, a1, a2, a3, xf[u][nt][1].x, xf[u][nt][1].y);
            }
            {
              const uint32_t a0 = lut_pair<2>(lut, wa[u].y, lane4), a2 = lut_pair<3>(lut, wa[u].y, lane4);
              const uint32_t a1 = lut_pair<2>(lut, wb[u].y, lane4), a3 = lut_pair<3>(lut, wb[u].y, lane4);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(p[nt], a0, a1, a2, a3, xf[u][nt][1].z, xf[u][nt][1].w);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[nt][0] = fmaf(p[nt][0], sa[u], acc[nt][0]);
              acc[nt][1] = fmaf(p[nt][1], sa[u], acc[nt][1]);
              acc[nt][2] = fmaf(p[nt][2], sb[u], acc[nt][2]);
              acc[nt][3] = fmaf(p[nt][3], sb[u], acc[nt][3]);
            }
          }
        }
      }
      // fixed-order reduction of the 8 K-slices
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) red[((warp * NT + nt) * 4 + r) * 32 + lane] = acc[nt][r];
      __syncthreads();
      if (warp == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float c[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) s += red[((w * NT + nt) * 4 + r) * 32 + lane];
            c[r] = s;
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int m = m0 + nt * 8 + 2 * q + h;
            if (m < M) {
              const int64_t srow = row0 + m;
              float va = c[h], vb = c[2 + h];
              if (g.a_scale) {
                const float sc = g.a_scale[g.a_rows ? g.a_rows[srow] : srow];
                va *= sc;
                vb *= sc;
              }
              if (g.rank) {
                va += lora_delta(g, e, rA, srow);
                vb += lora_delta(g, e, rB, srow);
              }
              OutT* o = reinterpret_cast<OutT*>(g.out) + srow * g.Nout;
              if (g.epilogue == E4B_EPI_SWIGLU) {
                o[tile * 8 + gq] = store_cast<OutT>(silu_f32(va) * vb, g.err);
              } else if (g.epilogue == E4B_EPI_SILU) {
                o[rA] = store_cast<OutT>(silu_f32(va), g.err);
                o[rB] = store_cast<OutT>(silu_f32(vb), g.err);
              } else {
                o[rA] = store_cast<OutT>(va, g.err);
                o[rB] = store_cast<OutT>(vb, g.err);
              }
            }
          }
        }
      }
      __syncthreads();
    }
  }
}

template <typename OutT, int NT>
static e4b_status launch_one(const GemvArgs& g, cudaStream_t s) {
  const int smem = kLutBytes + kGemvWarps * NT * 4 * 32 * (int)sizeof(float);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return E4B_ERR_CUDA;
  // the dynamic-smem opt-in is per device and per kernel instantiation
  static unsigned long long configured = 0;
  static int sm_count[64] = {0};
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    if (cudaFuncSetAttribute(nf4_gemv_kernel<OutT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return E4B_ERR_CUDA;
    cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    configured |= bit;
  }
  int grid = sm_count[dev & 63] * 3;
  if (g.max_tasks < grid) grid = g.max_tasks;
  if (grid < 1) return E4B_OK;
  nf4_gemv_kernel<OutT, NT><<<grid, kGemvThreads, smem, s>>>(g);
  return launch_status();
}

e4b_status launch_gemv(const GemvArgs& g, int max_rows_per_expert, cudaStream_t s) {
  const bool two = max_rows_per_expert > 8;
  if (g.out_dtype == E4B_BF16)
    return two ? launch_one<__nv_bfloat16, 2>(g, s) : launch_one<__nv_bfloat16, 1>(g, s);
  return two ? launch_one<__half, 2>(g, s) : launch_one<__half, 1>(g, s);
}

}  // namespace e4b
