// Streaming grouped NF4 GEMV for the decode regime (few tokens per expert).
//
// Same arithmetic as gemv.cu (fp16 code pairs from a lane-replicated table,
// mma.sync m16n8k16 with the activations as the n8 operand, fp32 per-block
// absmax scaling), organised for HBM bandwidth:
//  * one persistent CTA per SM builds the pair table once (32 KB: entry e of
//    lane l at (e << 7) | (l << 2), so no two lanes of a warp share a bank) and
//    stages the layer's activation rows in shared memory once;
//  * each of the 8 warps owns whole 16-row weight tiles (full K, no cross-warp
//    reduction) and streams them in 512-element chunks through its own
//    3-slot ring: lanes 0-15 bulk-copy one weight row each, lanes 16-31 the
//    matching absmax rows, completion tracked by one mbarrier per slot. Up to
//    3 x 4.6 KB are in flight per warp, ~100 KB per SM, independent of the
//    register file;
//  * shared-memory rows are padded (weights 288 B, absmax 48 B, activations
//    2K+16 B) so every fragment read is bank-conflict free.
// Waits are bounded; a timed-out wait reports E4B_ERR_TIMEOUT and the warp
// drains its in-flight copies (again bounded) before leaving.
#include "async.cuh"
#include "gemv.cuh"

namespace e4b {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kSlots = 3;
constexpr int kChunk = 512;                            // K elements per chunk
constexpr int kWPitch = kChunk / 2 + 32;               // 288 B per weight row (== 32 mod 128)
constexpr int kAPitch = 48;                            // absmax row: 8 floats + pad (bank spread)
constexpr int kSlotBytes = 16 * kWPitch + 16 * kAPitch;  // 5376
constexpr int kLut = 256 * 128;                        // 32 KB pair table
constexpr int kXBudget = 64 * 1024;                    // activation rows staged per CTA

struct Smem {
  static constexpr int lut = 0;
  static constexpr int x = kLut;
  static constexpr int slots = kLut + kXBudget;
  static constexpr int bars = slots + kWarps * kSlots * kSlotBytes;
  static constexpr int total = bars + kWarps * kSlots * 8;
};

__device__ __forceinline__ uint32_t lut2(const char* lut, uint32_t word, int pos, uint32_t lane4) {
  const uint32_t byte = (word >> (8 * pos)) & 0xffu;
  return *reinterpret_cast<const uint32_t*>(lut + ((byte << 7) | lane4));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Tile {
  int e, row0, M, tile;
};

__device__ __forceinline__ bool tile_of(const GemvArgs& g, int t, int num_active, Tile& out) {
  const int j = t / g.tiles_per_expert;
  if (t >= g.max_tasks || j >= num_active) return false;
  out.tile = t - j * g.tiles_per_expert;
  out.e = g.active[j];
  out.row0 = g.offsets[out.e];
  out.M = g.offsets[out.e + 1] - out.row0;
  return true;
}

// MMA row r (0..15) of a tile -> weight row.
__device__ __forceinline__ int weight_row(const GemvArgs& g, int tile, int r) {
  if (g.epilogue == E4B_EPI_SWIGLU) return r < 8 ? tile * 8 + r : (g.N >> 1) + tile * 8 + (r - 8);
  return tile * 16 + r;
}

}  // namespace

template <typename OutT, int NT>
__global__ void __launch_bounds__(kThreads, 1) nf4_gemv_stream_kernel(GemvArgs g, int x_rows) {
  extern __shared__ __align__(128) char smem[];
  char* lut = smem + Smem::lut;
  __half* xs = reinterpret_cast<__half*>(smem + Smem::x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  const int K = g.K;
  const int xpitch = K + 8;  // halves: 2K + 16 bytes
  char* myslots = smem + Smem::slots + warp * kSlots * kSlotBytes;
  uint64_t* mybars = reinterpret_cast<uint64_t*>(smem + Smem::bars) + warp * kSlots;

  if (lane == 0)
    for (int s = 0; s < kSlots; ++s) mbar_init(&mybars[s], 1);
  fence_proxy_async();
  __syncwarp();

  const int num_active = *g.num_active;
  const int nwarps = gridDim.x * kWarps;
  const int chunks = (K + kChunk - 1) / kChunk;

  // item n of this warp = (tile index n / chunks, chunk n % chunks)
  auto issue = [&](int n) {
    Tile tl;
    if (!tile_of(g, blockIdx.x * kWarps + warp + (n / chunks) * nwarps, num_active, tl)) return;
    const int c = n % chunks;
    const int kc = min(kChunk, K - c * kChunk);
    const int s = n % kSlots;
    char* slot = myslots + s * kSlotBytes;
    if (lane == 0) mbar_arrive_expect_tx(&mybars[s], 16u * (kc / 2) + 16u * (kc / 16));
    __syncwarp();
    const int r = lane & 15;
    const int64_t wrow = (int64_t)tl.e * g.N + weight_row(g, tl.tile, r);
    if (lane < 16) {
      bulk_g2s(slot + r * kWPitch, g.packed + wrow * (K / 2) + c * (kChunk / 2), kc / 2, &mybars[s]);
    } else {
      bulk_g2s(slot + 16 * kWPitch + r * kAPitch, g.absmax + wrow * (K / 64) + c * (kChunk / 64), kc / 16,
               &mybars[s]);
    }
  };

  // Prefetch the first items before the shared tables are built.
  int total_items = 0;
  {
    Tile tl;
    int tiles = 0;
    while (tile_of(g, blockIdx.x * kWarps + warp + tiles * nwarps, num_active, tl)) ++tiles;
    total_items = tiles * chunks;
  }
  for (int n = 0; n < kSlots && n < total_items; ++n) issue(n);

  // Pair table and activation rows (all threads).
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) {
    const int e = i >> 5, l = i & 31;
    reinterpret_cast<uint32_t*>(lut)[e * 32 + l] = pack2<__half>(c_nf4[e >> 4], c_nf4[e & 15]);
  }
  {
    const __half* A = reinterpret_cast<const __half*>(g.a);
    const int vec = K / 8;
    for (int i = threadIdx.x; i < x_rows * vec; i += blockDim.x) {
      const int r = i / vec, v = i - r * vec;
      *reinterpret_cast<uint4*>(xs + r * xpitch + v * 8) =
          *reinterpret_cast<const uint4*>(A + (int64_t)r * K + v * 8);
    }
  }
  __syncthreads();

  float acc[NT][4];
  bool ok = true;
  for (int n = 0; n < total_items; ++n) {
    const int c = n % chunks;
    Tile tl;
    tile_of(g, blockIdx.x * kWarps + warp + (n / chunks) * nwarps, num_active, tl);
    if (c == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
    }
    const int s = n % kSlots;
    if (!mbar_wait(&mybars[s], (n / kSlots) & 1)) {
      raise_error(g.err, E4B_ERR_TIMEOUT);
      // drain: items n .. n+kSlots-1 may still be in flight; wait for them (bounded) before leaving
      for (int m = n; m < n + kSlots && m < total_items; ++m) (void)mbar_wait(&mybars[m % kSlots], (m / kSlots) & 1);
      ok = false;
      break;
    }
    const char* slot = myslots + s * kSlotBytes;
    const int kc = min(kChunk, K - c * kChunk);
    // token rows of this tile's n8 column tiles (tokens >= M read row 0 and are discarded)
    const __half* xrow[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m = nt * 8 + gq;
      int src = 0;
      if (m < tl.M) src = g.a_rows ? g.a_rows[tl.row0 + m] : tl.row0 + m;
      xrow[nt] = xs + src * xpitch + c * kChunk + q * 16;
    }
#pragma unroll 2
    for (int b = 0; b < kc / 64; ++b) {
      const uint2 wa = *reinterpret_cast<const uint2*>(slot + gq * kWPitch + b * 32 + q * 8);
      const uint2 wb = *reinterpret_cast<const uint2*>(slot + (gq + 8) * kWPitch + b * 32 + q * 8);
      const float sa = *reinterpret_cast<const float*>(slot + 16 * kWPitch + gq * kAPitch + b * 4);
      const float sb = *reinterpret_cast<const float*>(slot + 16 * kWPitch + (gq + 8) * kAPitch + b * 4);
      uint4 xf[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        xf[nt][0] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64);
        xf[nt][1] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64 + 8);
      }
      float p[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) p[nt][r] = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const uint32_t w0 = jj < 2 ? wa.x : wa.y, w1 = jj < 2 ? wb.x : wb.y;
        const int p0 = (jj & 1) * 2;
        const uint32_t a0 = lut2(lut, w0, p0, lane4), a2 = lut2(lut, w0, p0 + 1, lane4);
        const uint32_t a1 = lut2(lut, w1, p0, lane4), a3 = lut2(lut, w1, p0 + 1, lane4);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xf[nt][jj >> 1]);
          mma16816(p[nt], a0, a1, a2, a3, xw[(jj & 1) * 2], xw[(jj & 1) * 2 + 1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[nt][0] = fmaf(p[nt][0], sa, acc[nt][0]);
        acc[nt][1] = fmaf(p[nt][1], sa, acc[nt][1]);
        acc[nt][2] = fmaf(p[nt][2], sb, acc[nt][2]);
        acc[nt][3] = fmaf(p[nt][3], sb, acc[nt][3]);
      }
    }
    // slot consumed: hand it back to the copy engine, refill with item n + kSlots
    fence_proxy_async();
    __syncwarp();
    if (n + kSlots < total_items) issue(n + kSlots);

    if (c == chunks - 1) {  // epilogue of the tile
      const int rA = weight_row(g, tl.tile, gq), rB = weight_row(g, tl.tile, gq + 8);
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
  (void)ok;
}

bool gemv_stream_eligible(const GemvArgs& g, int x_rows, int max_rows_per_expert) {
  return g.K % 256 == 0 && max_rows_per_expert <= 16 && (int64_t)x_rows * (g.K + 8) * 2 <= kXBudget &&
         g.epilogue >= E4B_EPI_NONE && g.epilogue <= E4B_EPI_SILU;
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
  const int need = (g.max_tasks + kWarps - 1) / kWarps;
  if (need < grid) grid = need;
  if (grid < 1) return E4B_OK;
  nf4_gemv_stream_kernel<OutT, NT><<<grid, kThreads, Smem::total, s>>>(g, x_rows);
  return launch_status();
}

e4b_status launch_gemv_stream(const GemvArgs& g, int x_rows, int max_rows_per_expert, cudaStream_t s) {
  const bool two = max_rows_per_expert > 8;
  if (g.out_dtype == E4B_BF16)
    return two ? launch_stream_one<__nv_bfloat16, 2>(g, x_rows, s) : launch_stream_one<__nv_bfloat16, 1>(g, x_rows, s);
  return two ? launch_stream_one<__half, 2>(g, x_rows, s) : launch_stream_one<__half, 1>(g, x_rows, s);
}

}  // namespace e4b
