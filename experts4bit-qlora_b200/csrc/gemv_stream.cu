// Streaming grouped NF4 GEMV for the decode regime (few tokens per expert).
//
// Same arithmetic as gemv.cu (fp16 code pairs from a lane-replicated table,
// mma.sync m16n8k16 with the activations as the n8 operand, fp32 per-block
// absmax scaling), organised for HBM bandwidth and short dependency chains:
//  * one persistent CTA per SM builds the pair table once (32 KB: entry e of
//    lane l at (e << 7) | (l << 2), so no two lanes of a warp share a bank) and
//    stages the layer's activation rows in shared memory once;
//  * the CTA's 16 warps form 8 pairs; a pair owns whole 16-row weight tiles
//    (full K) and streams them in 512-element chunks through its own 3-slot
//    ring, each warp of the pair taking half of every chunk's blocks and the
//    two halves summed through shared memory once per tile (fixed order). A
//    chunk is four TMA tile loads completing on one mbarrier: for each
//    8-row group, a 3-D box {128 B, 2 lines, 8 rows} of packed bytes with
//    128-byte swizzle, and a 2-D box {8 floats, 8 rows} of absmax. Because row
//    r of a group lands on shared-memory line 2r + c, the swizzle spreads the
//    eight rows of a half-warp over all banks: the fragment reads are
//    conflict free;
//  * a warp's four blocks of a chunk are unrolled with all packed words loaded
//    first, so the table lookups of different blocks overlap; a table address
//    is one shift and one lop3.
// Waits are bounded; a timed-out wait reports E4B_ERR_TIMEOUT and the warp
// drains its in-flight copies (again bounded) before leaving.
#include "stream_core.cuh"
#include "tmap.cuh"

// Profiling instrumentation, compiled only with -DE4B_TRACE: per-warp %globaltimer
// stamps at phase boundaries, read back with e4b_trace_read.
#ifdef E4B_TRACE
__device__ unsigned long long g_trace[148 * 8 * 8];
extern "C" __attribute__((visibility("default"))) int e4b_trace_read(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, g_trace, n * sizeof(unsigned long long));
}
#define TRACE(i)                                                     \
  if (lane == 0 && (warp & 1) == 0 && blockIdx.x < 148) {            \
    unsigned long long t_;                                           \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));          \
    g_trace[(blockIdx.x * 8 + (warp >> 1)) * 8 + (i)] = t_;          \
  }
#else
#define TRACE(i)
#endif

namespace e4b {

using namespace stream;

template <typename OutT, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_gemv_stream_kernel(GemvArgs g, int x_rows, const __grid_constant__ CUtensorMap wmap,
                           const __grid_constant__ CUtensorMap amap) {
  extern __shared__ __align__(1024) char smem[];
  char* lut = smem + Smem::lut;
  __half* xs = reinterpret_cast<__half*>(smem + Smem::x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int pair = warp >> 1, member = warp & 1;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  const int K = g.K;
  const int xpitch = K + 8;  // halves: 2K + 16 bytes
  char* myslots = smem + Smem::slots + pair * kSlots * kSlotBytes;
  float* red = reinterpret_cast<float*>(smem + Smem::red) + pair * 32 * 8;
  uint64_t* mybars = reinterpret_cast<uint64_t*>(smem + Smem::bars) + pair * kSlots;
  const bool leader = member == 0 && lane == 0;  // issues this pair's copies

  TRACE(0);
  // activation rows into registers first: their latency overlaps everything below
  const __half* A = reinterpret_cast<const __half*>(g.a);
  const int xvec = x_rows * (K / 8);
  uint4 xr[kXRegs];
#pragma unroll
  for (int i = 0; i < kXRegs; ++i) {
    const int v = threadIdx.x + i * kThreads;
    if (v < xvec) {
      const int r = v / (K / 8), c8 = v - r * (K / 8);
      xr[i] = *reinterpret_cast<const uint4*>(A + (int64_t)r * K + c8 * 8);
    }
  }
  if (leader) {
    for (int s = 0; s < kSlots; ++s) mbar_init(&mybars[s], 1);
    fence_proxy_async();
  }

  const int num_active = *g.num_active;
  const int npairs = gridDim.x * kPairs;
  const int chunks = (K + kChunk - 1) / kChunk;
  const int gp = blockIdx.x * kPairs + pair;
  // items of this pair in closed form: tiles gp, gp + npairs, ... below the limit, x chunks
  const int limit = min(g.max_tasks, num_active * g.tiles_per_expert);
  const int total_items = (limit > gp ? (limit - gp + npairs - 1) / npairs : 0) * chunks;

  auto issue = [&](int n) {  // leader only
    const int t = gp + (n / chunks) * npairs;
    const int j = t / g.tiles_per_expert;
    const int tile = t - j * g.tiles_per_expert;
    const int rowbase = g.active[j] * g.N;
    const int c = n % chunks;
    char* slot = myslots + (n % kSlots) * kSlotBytes;
    uint64_t* bar = &mybars[n % kSlots];
    mbar_arrive_expect_tx(bar, kItemTx);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r0 = rowbase + group_row(g, tile, h);
      tma_load_3d(slot + h * kBoxW, &wmap, 0, 2 * c, r0, bar);
      tma_load_2d(slot + 2 * kBoxW + h * kBoxA, &amap, 8 * c, r0, bar);
    }
  };

  TRACE(1);
  if (leader)
    for (int n = 0; n < kSlots && n < total_items; ++n) issue(n);
  TRACE(2);
  Tile tl;
  if (total_items > 0) tile_of(g, gp, tl);

  // Pair table (warp shuffles of the 16 codes), then the activation rows.
  {
    const float code = c_nf4[lane & 15];
#pragma unroll 4
    for (int e = warp; e < 256; e += kWarps) {
      const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
    }
#pragma unroll
    for (int i = 0; i < kXRegs; ++i) {
      const int v = threadIdx.x + i * kThreads;
      if (v < xvec) {
        const int r = v / (K / 8), c8 = v - r * (K / 8);
        *reinterpret_cast<uint4*>(xs + r * xpitch + c8 * 8) = xr[i];
      }
    }
  }
  __syncthreads();
  TRACE(3);

  float acc[NT][4];
  bool dead = false;  // a wait timed out: stop computing but keep the pair's barriers matched
  for (int n = 0; n < total_items; ++n) {
    const int c = n % chunks;
    if (c == 0) {
      if (n > 0) tile_of(g, gp + (n / chunks) * npairs, tl);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
    }
    const int s = n % kSlots;
    if (!dead && !mbar_wait(&mybars[s], (n / kSlots) & 1)) {
      raise_error(g.err, E4B_ERR_TIMEOUT);
      dead = true;
    }
    if (n == 0) TRACE(4);
    if (!dead) {
      const char* slot = myslots + s * kSlotBytes;
      const int nb = min(kChunk, K - c * kChunk) / 64;
      // token rows of this tile's n8 column tiles (tokens >= M read row 0 and are discarded)
      const __half* xrow[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + gq;
        int src = 0;
        if (m < tl.M) src = g.a_rows ? g.a_rows[tl.row0 + m] : tl.row0 + m;
        xrow[nt] = xs + src * xpitch + c * kChunk + q * 16;
      }
      // this member's blocks of the chunk: b = 4 * member + i (absmax floats 4*member..+3)
      const float4 sa4 = reinterpret_cast<const float4*>(slot + 2 * kBoxW + gq * 32)[member];
      const float4 sb4 = reinterpret_cast<const float4*>(slot + 2 * kBoxW + kBoxA + gq * 32)[member];
      const float sa[4] = {sa4.x, sa4.y, sa4.z, sa4.w}, sb[4] = {sb4.x, sb4.y, sb4.z, sb4.w};
      uint2 wa[4], wb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int b = 4 * member + i;
        wa[i] = *reinterpret_cast<const uint2*>(slot + wofs(smem_u32(slot), gq, q, b));
        wb[i] = *reinterpret_cast<const uint2*>(slot + kBoxW + wofs(smem_u32(slot + kBoxW), gq, q, b));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int b = 4 * member + i;
        if (b >= nb) break;
        uint4 xf[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          xf[nt][0] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64);
          xf[nt][1] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64 + 8);
        }
        float p[NT][4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t w0 = jj < 2 ? wa[i].x : wa[i].y, w1 = jj < 2 ? wb[i].x : wb[i].y;
          uint32_t a0, a1, a2, a3;
          if (jj & 1) {
            a0 = lut2<2>(lut, w0, lane4); a2 = lut2<3>(lut, w0, lane4);
            a1 = lut2<2>(lut, w1, lane4); a3 = lut2<3>(lut, w1, lane4);
          } else {
            a0 = lut2<0>(lut, w0, lane4); a2 = lut2<1>(lut, w0, lane4);
            a1 = lut2<0>(lut, w1, lane4); a3 = lut2<1>(lut, w1, lane4);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xf[nt][jj >> 1]);
            if (jj == 0)
              mma16816_zero(p[nt], a0, a1, a2, a3, xw[0], xw[1]);
            else
              mma16816(p[nt], a0, a1, a2, a3, xw[(jj & 1) * 2], xw[(jj & 1) * 2 + 1]);
          }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[nt][0] = fmaf(p[nt][0], sa[i], acc[nt][0]);
          acc[nt][1] = fmaf(p[nt][1], sa[i], acc[nt][1]);
          acc[nt][2] = fmaf(p[nt][2], sb[i], acc[nt][2]);
          acc[nt][3] = fmaf(p[nt][3], sb[i], acc[nt][3]);
        }
      }
    }
    const bool last = c == chunks - 1;
    if (last && member == 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) red[(nt * 4 + r) * 32 + lane] = acc[nt][r];
    }
    // both members are done with the slot (and member 1's partial sums are written); the proxy
    // fence orders their generic reads before the slot's refill by the async proxy
    fence_proxy_async();
    named_barrier(1 + pair, 64);
    if (n == 0) TRACE(5);
    if (leader && !dead && n + kSlots < total_items) issue(n + kSlots);
    if (n == 0) TRACE(7);

    if (last && member == 0 && !dead) {  // epilogue of the tile
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] += red[(nt * 4 + r) * 32 + lane];
      const int rA = group_row(g, tl.tile, 0) + gq, rB = group_row(g, tl.tile, 1) + gq;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m = nt * 8 + 2 * q + h;
          if (m >= tl.M) continue;
          const int64_t srow = tl.row0 + m;
          float va = acc[nt][h], vb = acc[nt][2 + h];
          if (g.a_scale) {
            const float sc = g.a_scale[g.a_rows ? g.a_rows[srow] : srow];
            va *= sc;
            vb *= sc;
          }
          if (g.rank) {
            const float* xa = g.lora_xa + srow * g.rank;
            const int64_t ba = ((int64_t)tl.e * g.N + rA) * g.rank, bb = ((int64_t)tl.e * g.N + rB) * g.rank;
            for (int j = 0; j < g.rank; ++j) {
              va = fmaf(xa[j], load_as_f32(g.lora_B, g.lora_dtype, ba + j), va);
              vb = fmaf(xa[j], load_as_f32(g.lora_B, g.lora_dtype, bb + j), vb);
            }
          }
          OutT* o = reinterpret_cast<OutT*>(g.out) + srow * g.Nout;
          if (g.epilogue == E4B_EPI_SWIGLU) {
            o[tl.tile * 8 + gq] = store_cast<OutT>(silu_f32(va) * vb, g.err);
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
  if (dead && leader) {
    // drain (bounded) whatever may still be in flight before the CTA's shared memory goes away
    for (int m = 0; m < total_items && m < kSlots; ++m) (void)mbar_wait(&mybars[m], 0);
  }
  TRACE(6);
}

bool gemv_stream_eligible(const GemvArgs& g, int x_rows, int max_rows_per_expert) {
  return g.K % 256 == 0 && max_rows_per_expert <= 16 && (int64_t)x_rows * (g.K + 8) * 2 <= kXBudget &&
         g.epilogue >= E4B_EPI_NONE && g.epilogue <= E4B_EPI_SILU && (int64_t)g.E * g.N < (1ll << 31) &&
         encode_tiled_fn() != nullptr;
}

template <typename OutT, int NT>
static e4b_status launch_stream_one(const GemvArgs& g, int x_rows, cudaStream_t s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return E4B_ERR_CUDA;
  static unsigned long long configured = 0;
  static int sm_count[64] = {0};
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    if (cudaFuncSetAttribute(nf4_gemv_stream_kernel<OutT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Smem::total) != cudaSuccess)
      return E4B_ERR_CUDA;
    cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    configured |= bit;
  }
  int grid = sm_count[dev & 63];
  const int need = (g.max_tasks + kPairs - 1) / kPairs;
  if (need < grid) grid = need;
  if (grid < 1) return E4B_OK;
  // packed bytes as [rows][K/256 lines][128 B]; absmax as [rows][K/64]
  const cuuint64_t rows = (cuuint64_t)g.E * g.N;
  CUtensorMap wmap, amap;
  const cuuint64_t wdims[3] = {128, (cuuint64_t)(g.K / 256), rows};
  const cuuint64_t wstr[2] = {128, (cuuint64_t)(g.K / 2)};
  const cuuint32_t wbox[3] = {128, 2, 8};
  const cuuint64_t adims[2] = {(cuuint64_t)(g.K / 64), rows};
  const cuuint64_t astr[1] = {(cuuint64_t)(g.K / 64) * 4};
  const cuuint32_t abox[2] = {8, 8};
  if (!encode_tiled(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, g.packed, wdims, wstr, wbox,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_tiled(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, g.absmax, adims, astr, abox,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
    return E4B_ERR_CUDA;
  nf4_gemv_stream_kernel<OutT, NT><<<grid, kThreads, Smem::total, s>>>(g, x_rows, wmap, amap);
  return launch_status();
}

e4b_status launch_gemv_stream(const GemvArgs& g, int x_rows, int max_rows_per_expert, cudaStream_t s) {
  const bool two = max_rows_per_expert > 8;
  if (g.out_dtype == E4B_BF16)
    return two ? launch_stream_one<__nv_bfloat16, 2>(g, x_rows, s) : launch_stream_one<__nv_bfloat16, 1>(g, x_rows, s);
  return two ? launch_stream_one<__half, 2>(g, x_rows, s) : launch_stream_one<__half, 1>(g, x_rows, s);
}

}  // namespace e4b
