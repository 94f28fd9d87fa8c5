// Block-scaled FP8 expert weights: the dequant entry point and the grouped
// GEMV of the decode regime.
//
// Storage follows formats/fp8_blocks.py:60-128: e4m3 bytes [out, in] with one
// multiplier per [128, 128] tile. The reference has no fused FP8 expert path:
// its semantics are the per-expert loop (_vendor/experts.py:468-516) over
// dequantize_fp8_blocks weights, W = bf16(fp32(w) * scale), then a bf16 matmul.
// The fused kernels keep the weights at full precision instead (e4m3 -> fp16 is
// exact; the fp32 tile scale multiplies fp32 partial sums, or a power-of-two
// ratio of it is folded into the fp16 operand) and share the NF4 path's fp16
// activations with per-row power-of-two scales and fp16 intermediates: the bf16
// rounding of the intermediate activation in the reference loop alone costs about
// 4e-3 of mean relative error against the fp32 result.
#include "fp8.cuh"
#include "gemv.cuh"

namespace e4b {

namespace {

template <typename OutT>
__global__ void __launch_bounds__(256) fp8_dequant_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale,
                                                          int64_t rows, int64_t cols, int aligned,
                                                          OutT* __restrict__ out) {
  // Aligned shapes take formats/fp8_blocks.py's aligned path, which multiplies in the
  // output dtype: the scale is rounded to it first (a no-op for e8m0 scales).
  const auto eff = [&](float v) { return aligned ? to_f32<OutT>(from_f32<OutT>(v)) : v; };
  const int64_t tiles_in = (cols + kFp8Block - 1) / kFp8Block;
  const int64_t n = rows * cols;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((cols & 7) == 0) {  // 8 elements per step; a group never crosses a tile edge
    const int64_t groups = n / 8;
    for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += stride) {
      const int64_t i0 = gi * 8, o = i0 / cols, c = i0 - o * cols;
      const float s = eff(scale[(o / kFp8Block) * tiles_in + c / kFp8Block]);
      const uint2 b = *reinterpret_cast<const uint2*>(w + i0);
      const uint32_t words[2] = {b.x, b.y};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float2 lo = e4m3x2_to_f32x2(words[j] & 0xffffu), hi = e4m3x2_to_f32x2(words[j] >> 16);
        out[i0 + 4 * j + 0] = from_f32<OutT>(lo.x * s);
        out[i0 + 4 * j + 1] = from_f32<OutT>(lo.y * s);
        out[i0 + 4 * j + 2] = from_f32<OutT>(hi.x * s);
        out[i0 + 4 * j + 3] = from_f32<OutT>(hi.y * s);
      }
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t o = i / cols, c = i - o * cols;
    const float s = eff(scale[(o / kFp8Block) * tiles_in + c / kFp8Block]);
    out[i] = from_f32<OutT>(e4m3x2_to_f32x2(w[i]).x * s);
  }
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// One warp per task = (active expert, 16-row feature tile); all K; the expert's
// tokens in groups of 16 (two n8 MMA tiles). fp16 MMAs: A = fp16(e4m3), exact;
// B = the fp16 activation rows (per-row power-of-two scale, convert.cuh). Each
// 128-wide K block accumulates into fp32 partials that are folded in with the
// block's scale, so the weights enter at full fp32 scale precision; the token's
// activation scale is applied in the epilogue. K is permuted consistently for A
// and B inside each 64-element chunk: lane q of a quad holds bytes 16q..16q+15 of
// the chunk, and k-step j uses its bytes 4j..4j+3 as the fragment's {2q, 2q+1,
// 2q+8, 2q+9} columns, so a lane loads 16 contiguous weight bytes per row and 32
// contiguous activation bytes per token per chunk. For SwiGLU the warp
// accumulates the gate and up tiles of the same features side by side.
template <typename OutT, int GROUPS>
__global__ void __launch_bounds__(256) fp8_gemv_kernel(GemvArgs g) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, q = lane & 3;
  const int tiles = g.tiles_per_expert;
  const int ntask = *g.num_active * tiles;
  const int Nh = GROUPS == 2 ? g.N / 2 : g.N;
  const int kchunks = g.K / 64;
  const int kblocks = g.K / kFp8Block;
  const __half* __restrict__ x = reinterpret_cast<const __half*>(g.a);
  for (int task = blockIdx.x * 8 + (threadIdx.x >> 5); task < ntask; task += gridDim.x * 8) {
    const int ai = task / tiles, rt = task - ai * tiles;
    const int e = g.active[ai];
    const int row0 = g.offsets[e], cnt = g.offsets[e + 1] - row0;
    const int frow = rt * 16;
    const uint8_t* wr[GROUPS][2];
    const float* sc[GROUPS];
#pragma unroll
    for (int h = 0; h < GROUPS; ++h) {
      const int row = (h == 0 ? 0 : Nh) + frow;
      const uint8_t* base = g.packed + ((int64_t)e * g.N + row) * g.K + 16 * q;
      wr[h][0] = base + (int64_t)gq * g.K;
      wr[h][1] = base + (int64_t)(gq + 8) * g.K;
      sc[h] = g.absmax + ((int64_t)e * (g.N / kFp8Block) + row / kFp8Block) * kblocks;
    }
    for (int tok0 = 0; tok0 < cnt; tok0 += 16) {
      const int t0 = tok0 + gq, t1 = tok0 + 8 + gq;
      const bool two = cnt - tok0 > 8;
      const __half* x0 = nullptr;
      const __half* x1 = nullptr;
      if (t0 < cnt) x0 = x + (int64_t)(g.a_rows ? g.a_rows[row0 + t0] : row0 + t0) * g.K + 16 * q;
      if (t1 < cnt) x1 = x + (int64_t)(g.a_rows ? g.a_rows[row0 + t1] : row0 + t1) * g.K + 16 * q;
      float acc[GROUPS][2][4], part[GROUPS][2][4];
#pragma unroll
      for (int h = 0; h < GROUPS; ++h)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[h][nt][i] = part[h][nt][i] = 0.f;
      uint4 wcur[GROUPS][2];
#pragma unroll
      for (int h = 0; h < GROUPS; ++h) {
        wcur[h][0] = ldg_nc_u4(wr[h][0]);
        wcur[h][1] = ldg_nc_u4(wr[h][1]);
      }
      for (int c = 0; c < kchunks; ++c) {
        uint4 wnext[GROUPS][2];
        if (c + 1 < kchunks) {
#pragma unroll
          for (int h = 0; h < GROUPS; ++h) {
            wnext[h][0] = ldg_nc_u4(wr[h][0] + (c + 1) * 64);
            wnext[h][1] = ldg_nc_u4(wr[h][1] + (c + 1) * 64);
          }
        }
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 xa0 = x0 ? *reinterpret_cast<const uint4*>(x0 + c * 64) : z;
        const uint4 xb0 = x0 ? *reinterpret_cast<const uint4*>(x0 + c * 64 + 8) : z;
        uint4 xa1 = z, xb1 = z;
        if (two && x1) {
          xa1 = *reinterpret_cast<const uint4*>(x1 + c * 64);
          xb1 = *reinterpret_cast<const uint4*>(x1 + c * 64 + 8);
        }
        const uint32_t bt0[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xb0.x, xb0.y, xb0.z, xb0.w};
        const uint32_t bt1[8] = {xa1.x, xa1.y, xa1.z, xa1.w, xb1.x, xb1.y, xb1.z, xb1.w};
#pragma unroll
        for (int h = 0; h < GROUPS; ++h) {
          const uint32_t r0[4] = {wcur[h][0].x, wcur[h][0].y, wcur[h][0].z, wcur[h][0].w};
          const uint32_t r1[4] = {wcur[h][1].x, wcur[h][1].y, wcur[h][1].z, wcur[h][1].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a0 = e4m3x2_to_f16x2(r0[j] & 0xffffu);
            const uint32_t a2 = e4m3x2_to_f16x2(r0[j] >> 16);
            const uint32_t a1 = e4m3x2_to_f16x2(r1[j] & 0xffffu);
            const uint32_t a3 = e4m3x2_to_f16x2(r1[j] >> 16);
            mma_f16(part[h][0], a0, a1, a2, a3, bt0[2 * j], bt0[2 * j + 1]);
            if (two) mma_f16(part[h][1], a0, a1, a2, a3, bt1[2 * j], bt1[2 * j + 1]);
          }
          if (c & 1) {  // end of a 128-wide K block: fold the partials in with its scale
            const float s = __ldg(sc[h] + (c >> 1));
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                acc[h][nt][i] = fmaf(s, part[h][nt][i], acc[h][nt][i]);
                part[h][nt][i] = 0.f;
              }
          }
        }
        if (c + 1 < kchunks) {
#pragma unroll
          for (int h = 0; h < GROUPS; ++h) {
            wcur[h][0] = wnext[h][0];
            wcur[h][1] = wnext[h][1];
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tok = tok0 + nt * 8 + 2 * q + (i & 1);
          if (tok >= cnt) continue;
          const int srow = row0 + tok;
          const float ts = g.a_scale ? g.a_scale[g.a_rows ? g.a_rows[srow] : srow] : 1.f;
          const int feat = frow + gq + (i >> 1) * 8;
          float v = acc[0][nt][i] * ts;
          if (GROUPS == 2)
            v = silu_f32(v) * (acc[GROUPS - 1][nt][i] * ts);
          else if (g.epilogue == E4B_EPI_SILU)
            v = silu_f32(v);
          reinterpret_cast<OutT*>(g.out)[(int64_t)srow * g.Nout + feat] = store_cast<OutT>(v, g.err);
        }
    }
  }
}

template <typename OutT>
e4b_status launch_fp8_dequant(const uint8_t* w, const float* scale, int64_t rows, int64_t cols, void* out,
                              cudaStream_t s) {
  const int64_t n = rows * cols;
  const int64_t work = (cols & 7) == 0 ? n / 8 : n;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  const int aligned = rows % kFp8Block == 0 && cols % kFp8Block == 0;
  fp8_dequant_kernel<OutT><<<(unsigned)blocks, 256, 0, s>>>(w, scale, rows, cols, aligned, static_cast<OutT*>(out));
  return launch_status();
}

}  // namespace

e4b_status launch_fp8_gemv(const GemvArgs& g, cudaStream_t s) {
  if (g.K % kFp8Block || g.N % (g.epilogue == E4B_EPI_SWIGLU ? 2 * kFp8Block : kFp8Block)) return E4B_ERR_UNSUPPORTED;
  int blocks = (g.max_tasks + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) return E4B_OK;
  const bool two = g.epilogue == E4B_EPI_SWIGLU;
  if (g.out_dtype == E4B_BF16) {
    if (two) fp8_gemv_kernel<__nv_bfloat16, 2><<<blocks, 256, 0, s>>>(g);
    else fp8_gemv_kernel<__nv_bfloat16, 1><<<blocks, 256, 0, s>>>(g);
  } else {
    if (two) fp8_gemv_kernel<__half, 2><<<blocks, 256, 0, s>>>(g);
    else fp8_gemv_kernel<__half, 1><<<blocks, 256, 0, s>>>(g);
  }
  return launch_status();
}

}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_fp8_block_dequantize(const uint8_t* w, const float* scale, int64_t rows, int64_t cols,
                                               void* out, int out_dtype, void* stream) {
  if (rows < 0 || cols < 0) return E4B_ERR_INVALID_ARG;
  if (!is_any_dtype(out_dtype)) return E4B_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return E4B_OK;
  if (!w || !scale || !out) return E4B_ERR_INVALID_ARG;
  if ((cols & 7) == 0 && (reinterpret_cast<uintptr_t>(w) & 7)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  switch (out_dtype) {
    case E4B_BF16: return launch_fp8_dequant<__nv_bfloat16>(w, scale, rows, cols, out, s);
    case E4B_F16: return launch_fp8_dequant<__half>(w, scale, rows, cols, out, s);
    default: return launch_fp8_dequant<float>(w, scale, rows, cols, out, s);
  }
}
