// LoRA-A pre-pass (R5): xa[r, :] = scaling * (a_r . A[e]^T) for every sorted row r
// of expert e -- the first factor of ExpertsLoRA._lora (experts4bit_qlora/lora.py:
// 251-256); the second factor (. B[e]^T) and the add before the activation are
// fused into the grouped GEMM epilogues.
//
// A CTA takes 64 rows of one expert; each of its 4 warps computes 16 rows x all
// ranks with mma.sync m16n8k16 (fp16 operands, fp32 accumulation), the 64-wide K
// chunks of the rows and of A[e] staged in padded shared memory.
#include <cstdlib>

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

namespace {
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {  // bytes 0: zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Eight adapter values (lora dtype) from 16-byte-aligned storage as fp16, rounded like
// __float2half_rn(load_as_f32(...)) element by element.
__device__ __forceinline__ uint4 lora8_as_f16(const void* base, int dtype, int64_t i) {
  uint32_t o[4];
  if (dtype == E4B_F32) {
    const float4 lo = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
    const float4 hi = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i + 4);
    o[0] = pack2<__half>(lo.x, lo.y);
    o[1] = pack2<__half>(lo.z, lo.w);
    o[2] = pack2<__half>(hi.x, hi.y);
    o[3] = pack2<__half>(hi.z, hi.w);
  } else {
    const uint4 r = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + i);
    if (dtype == E4B_F16) return r;
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack2<__half>(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xffff0000u));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
}  // namespace

// The same products as lora_a_kernel (same fragments, same K order, so bit-identical) for ranks
// <= 16 with 128-wide K chunks double-buffered: the next chunk's activation rows (cp.async) and
// adapter rows (16-byte loads, converted in registers) are in flight while the tensor cores work
// on this chunk; one barrier per chunk.
template <int NR>
__global__ void __launch_bounds__(128) lora_a_pipe_kernel(LoraAArgs g) {
  constexpr int kKc = 128;
  constexpr int kPitch = kKc + 8;  // 272-byte rows: 16-byte aligned, conflict-free fragment reads
  __shared__ __align__(16) __half xs[2][kLoraRows][kPitch];
  __shared__ __align__(16) __half as[2][8 * NR][kPitch];
  const int t = blockIdx.x;
  if (t >= g.tile_start[g.E]) return;
  int lo = 0, hi = g.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (g.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int e = lo;
  const int r0 = g.offsets[e] + (t - g.tile_start[e]) * kLoraRows;
  const int rend = g.offsets[e + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, q = lane & 3;
  const int nch = (g.K + kKc - 1) / kKc;
  // this thread's activation rows (source rows fixed over the chunks)
  int64_t srow[kLoraRows * (kKc / 8) / 128];
#pragma unroll
  for (int u = 0; u < kLoraRows * (kKc / 8) / 128; ++u) {
    const int r = r0 + ((threadIdx.x + 128 * u) >> 4);
    srow[u] = r < rend ? (g.a_rows ? (int64_t)g.a_rows[r] : (int64_t)r) : -1;
  }
  auto issue_x = [&](int c, int buf) {
    const int k0 = c * kKc;
#pragma unroll
    for (int u = 0; u < kLoraRows * (kKc / 8) / 128; ++u) {
      const int i = threadIdx.x + 128 * u, rr = i >> 4, v = i & 15;
      const bool ok = srow[u] >= 0 && k0 + v * 8 < g.K;
      const __half* src = ok ? g.a + srow[u] * g.K + k0 + v * 8 : g.a;
      cp_async16(&xs[buf][rr][v * 8], src, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  auto load_a = [&](int c, uint4 (&av)[NR]) {
    const int k0 = c * kKc;
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      const int i = threadIdx.x + 128 * u, j = i >> 4, v = i & 15;
      av[u] = (j < g.rank && k0 + v * 8 < g.K)
                  ? lora8_as_f16(g.loraA, g.lora_dtype, ((int64_t)e * g.rank + j) * g.K + k0 + v * 8)
                  : make_uint4(0, 0, 0, 0);
    }
  };
  auto store_a = [&](int buf, const uint4 (&av)[NR]) {
#pragma unroll
    for (int u = 0; u < NR; ++u) {
      const int i = threadIdx.x + 128 * u;
      *reinterpret_cast<uint4*>(&as[buf][i >> 4][(i & 15) * 8]) = av[u];
    }
  };
  float acc[NR][4];
#pragma unroll
  for (int n = 0; n < NR; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
  uint4 av[NR];
  issue_x(0, 0);
  load_a(0, av);
  store_a(0, av);
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    cp_async_wait_all();
    __syncthreads();  // chunk c visible; every warp is done with chunk c - 1 (the other buffer)
    if (c + 1 < nch) {
      issue_x(c + 1, buf ^ 1);
      load_a(c + 1, av);
    }
#pragma unroll
    for (int ks = 0; ks < kKc; ks += 16) {
      const int rw = warp * 16 + gq;
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw][ks + 2 * q]);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw + 8][ks + 2 * q]);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw][ks + 2 * q + 8]);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw + 8][ks + 2 * q + 8]);
#pragma unroll
      for (int n = 0; n < NR; ++n) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&as[buf][n * 8 + gq][ks + 2 * q]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&as[buf][n * 8 + gq][ks + 2 * q + 8]);
        mma_f16(acc[n], a0, a1, a2, a3, b0, b1);
      }
    }
    if (c + 1 < nch) store_a(buf ^ 1, av);  // nobody reads that buffer until the next barrier
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + warp * 16 + gq + 8 * h;
    if (r >= rend) continue;
    if (g.xa16) {
#pragma unroll
      for (int n = 0; n < NR; ++n) {
        const int j = n * 8 + 2 * q;
        *reinterpret_cast<__half2*>(g.xa16 + (int64_t)r * 64 + j) =
            __floats2half2_rn(j < g.rank ? g.scaling * acc[n][2 * h] : 0.f,
                              j + 1 < g.rank ? g.scaling * acc[n][2 * h + 1] : 0.f);
      }
      if (NR == 1) *reinterpret_cast<__half2*>(g.xa16 + (int64_t)r * 64 + 8 + 2 * q) = __floats2half2_rn(0.f, 0.f);
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
  // pipelined kernel: ranks <= 16, 16-byte aligned activation and adapter storage (E4B_LORA_A_PIPE=0: off)
  static const bool pipe = [] {
    const char* v = getenv("E4B_LORA_A_PIPE");
    return !(v && v[0] == '0');
  }();
  if (pipe && nr <= 2 && !((uintptr_t)g.a & 15) && !((uintptr_t)g.loraA & 15)) {
    if (nr <= 1)
      lora_a_pipe_kernel<1><<<g.max_tiles, 128, 0, s>>>(g);
    else
      lora_a_pipe_kernel<2><<<g.max_tiles, 128, 0, s>>>(g);
    return launch_status();
  }
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
