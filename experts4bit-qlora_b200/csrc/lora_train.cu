// Rank-r adapter products of the training path (train.py; reference engines/fast.py:453-552 and
// lora.py:251-256) over expert-sorted rows, in fp32 on the CUDA cores, with no padding of the
// experts' row segments:
//   rank-down   Y[row, j]  = scale * sum_k X[row, k] * M_e(j, k)          (x . A^T, dD . B, h . A^T)
//   rank-up     Z[row, n] (+)= scale * sum_j Y[row, j] * M_e(j, n)       (xa . B^T, t . A)
//   outer       G_e(a, j)  = scale * sum_{rows of e} P[row, a] * Y[row, j]  (the adapter gradients)
// M_e(j, k) = M[e * sE + j * sj + k * sk]: the same kernels read A [E, r, K] and B [E, N, r]
// in either orientation. The row tiles (expert, first row, rows) come from the host, which knows
// the experts' row counts already (the training forward's one sync). Ranks up to 16. Every sum
// has a fixed order, so results repeat bit for bit.
#include <type_traits>

#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace e4b {
namespace {

constexpr int kRk = 16;     // rank slots per row (ranks below 16 leave the rest unused)
constexpr int kTileR = 32;  // rows per tile
constexpr int kKc = 256;    // K elements per staged chunk of M

__device__ __forceinline__ void cp_async4(void* dst, const void* src, int bytes) {  // bytes 0: zero fill
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(bytes)
               : "memory");
}

// Shared memory of rank_down_kernel: two stages of the M chunk (fp32) and of the tile's X rows.
template <typename TX>
constexpr int rank_down_smem() {
  return 2 * kRk * kKc * 4 + 2 * kTileR * kKc * (int)sizeof(TX);
}

template <typename TX>
__global__ void __launch_bounds__(256) rank_down_kernel(const TX* __restrict__ X, int ldx, const float* __restrict__ M,
                                                        int64_t sE, int64_t sj, int64_t sk, int rk, int K,
                                                        const int* __restrict__ tiles, float scale,
                                                        float* __restrict__ Y) {
  // Double-buffered over K chunks: the next chunk's M values and X rows are copied into shared
  // memory by cp.async while this chunk's FMAs run, one barrier per chunk. Every lane accumulates
  // its k in the same order as a one-buffer loop.
  extern __shared__ __align__(16) char smem_raw[];
  float (*ms)[kRk][kKc] = reinterpret_cast<float (*)[kRk][kKc]>(smem_raw);
  TX (*xs)[kTileR][kKc] = reinterpret_cast<TX (*)[kTileR][kKc]>(smem_raw + 2 * kRk * kKc * 4);
  const int e = tiles[blockIdx.x * 3], row0 = tiles[blockIdx.x * 3 + 1], nrows = tiles[blockIdx.x * 3 + 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float acc[4][kRk];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < kRk; ++j) acc[r][j] = 0.f;
  const float* Me = M + (int64_t)e * sE;
  const bool m_vec = sk == 1 && (sj & 3) == 0 && ((uintptr_t)Me & 15) == 0;  // 16-byte M copies
  constexpr int kXv = kKc * (int)sizeof(TX) / 16;                           // 16-byte vectors per X row
  auto issue = [&](int kc, int buf) {
    if (m_vec) {
      for (int i = threadIdx.x; i < kRk * kKc / 4; i += 256) {
        const int j = i / (kKc / 4), c = (i - j * (kKc / 4)) * 4;
        const bool ok = j < rk && kc + c < K;  // K % 8 == 0: a vector is all in or all out
        cp_async16(&ms[buf][j][c], ok ? Me + j * sj + kc + c : Me, ok ? 16 : 0);
      }
    } else {
      for (int i = threadIdx.x; i < kRk * kKc; i += 256) {
        const int j = i / kKc, c = i - j * kKc;
        const bool ok = j < rk && kc + c < K;
        cp_async4(&ms[buf][j][c], ok ? Me + j * sj + (int64_t)(kc + c) * sk : Me, ok ? 4 : 0);
      }
    }
    for (int i = threadIdx.x; i < kTileR * kXv; i += 256) {
      const int rr = i / kXv, v = i - rr * kXv;
      const int c = v * (16 / (int)sizeof(TX));
      const bool ok = rr < nrows && kc + c < K;
      cp_async16(&xs[buf][rr][c], ok ? X + (int64_t)(row0 + rr) * ldx + kc + c : X, ok ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const int kk = lane * 8;  // lane owns 8 consecutive k of a chunk
  issue(0, 0);
  for (int kc = 0, buf = 0; kc < K; kc += kKc, buf ^= 1) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // chunk kc visible; every thread is done with the other buffer
    if (kc + kKc < K) issue(kc + kKc, buf ^ 1);
    if (kc + kk < K) {
      float xv[4][8];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const TX* xp = &xs[buf][warp * 4 + r][kk];
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[r][i] = to_f32(xp[i]);
      }
#pragma unroll
      for (int j = 0; j < kRk; ++j) {
        const float4 m0 = *reinterpret_cast<const float4*>(&ms[buf][j][kk]);
        const float4 m1 = *reinterpret_cast<const float4*>(&ms[buf][j][kk + 4]);
        const float m[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[r][j] = fmaf(xv[r][i], m[i], acc[r][j]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int rr = warp * 4 + r;
#pragma unroll
    for (int j = 0; j < kRk; ++j) {
      float v = acc[r][j];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == j && j < rk && rr < nrows) Y[(int64_t)(row0 + rr) * rk + j] = v * scale;
    }
  }
}

// bf16 rows on the tensor cores: M (fp32) is split per chunk into three bf16 parts
// (hi = bf16(M), mid = bf16(M - hi), lo = bf16(M - hi - mid), which sum to M within about 2^-24
// relative), and each part multiplies the bf16 rows exactly (mma.sync m16n8k16, fp32
// accumulation), so Y keeps fp32 accuracy at a fraction of the CUDA-core cost. Two warps per
// 32-row tile, 16 rows each, all 16 rank slots (two n8 tiles); 128-wide K chunks of X arrive by
// cp.async and of M by registers, both double-buffered with one barrier per chunk.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kMc = 128;         // K per chunk of the tensor-core kernel
constexpr int kMp = kMc + 8;     // padded row (halves): conflict-free fragment reads
constexpr int kMPer = kRk * kMc / 64;  // M values per thread per chunk

__global__ void __launch_bounds__(64) rank_down_mma_kernel(const __nv_bfloat16* __restrict__ X, int ldx,
                                                           const float* __restrict__ M, int64_t sE, int64_t sj,
                                                           int64_t sk, int rk, int K, const int* __restrict__ tiles,
                                                           float scale, float* __restrict__ Y) {
  __shared__ __align__(16) __nv_bfloat16 xs[2][kTileR][kMp];
  __shared__ __align__(16) __nv_bfloat16 m3[2][3][kRk][kMp];
  const int e = tiles[blockIdx.x * 3], row0 = tiles[blockIdx.x * 3 + 1], nrows = tiles[blockIdx.x * 3 + 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const float* Me = M + (int64_t)e * sE;
  float mr[kMPer];
  auto issue_x = [&](int kc, int buf) {
#pragma unroll
    for (int u = 0; u < kTileR * (kMc / 8) / 64; ++u) {
      const int i = threadIdx.x + 64 * u, rr = i / (kMc / 8), c = (i % (kMc / 8)) * 8;
      const bool ok = rr < nrows && kc + c < K;
      cp_async16(&xs[buf][rr][c], ok ? X + (int64_t)(row0 + rr) * ldx + kc + c : X, ok ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto load_m = [&](int kc) {
#pragma unroll
    for (int u = 0; u < kMPer; ++u) {
      const int i = threadIdx.x + 64 * u, j = i / kMc, c = i % kMc;
      mr[u] = (j < rk && kc + c < K) ? Me[j * sj + (int64_t)(kc + c) * sk] : 0.f;
    }
  };
  auto store_m = [&](int buf) {
#pragma unroll
    for (int u = 0; u < kMPer; ++u) {
      const int i = threadIdx.x + 64 * u, j = i / kMc, c = i % kMc;
      const float v = mr[u];
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const float r1 = v - __bfloat162float(hi);
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
      m3[buf][0][j][c] = hi;
      m3[buf][1][j][c] = mid;
      m3[buf][2][j][c] = lo;
    }
  };
  float acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
  issue_x(0, 0);
  load_m(0);
  store_m(0);
  for (int kc = 0, buf = 0; kc < K; kc += kMc, buf ^= 1) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // chunk kc visible; both warps are done with the other buffers
    const bool more = kc + kMc < K;
    if (more) {
      issue_x(kc + kMc, buf ^ 1);
      load_m(kc + kMc);
    }
    const int rw = warp * 16 + g;
#pragma unroll
    for (int ks = 0; ks < kMc; ks += 16) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw][ks + 2 * q]);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw + 8][ks + 2 * q]);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw][ks + 2 * q + 8]);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(&xs[buf][rw + 8][ks + 2 * q + 8]);
#pragma unroll
      for (int p = 2; p >= 0; --p)  // smallest part first
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&m3[buf][p][n * 8 + g][ks + 2 * q]);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&m3[buf][p][n * 8 + g][ks + 2 * q + 8]);
          mma_bf16(acc[n], a0, a1, a2, a3, b0, b1);
        }
    }
    if (more) store_m(buf ^ 1);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rr = warp * 16 + g + 8 * h;
    if (rr >= nrows) continue;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int j = n * 8 + 2 * q + c;
        if (j < rk) Y[(int64_t)(row0 + rr) * rk + j] = acc[n][2 * h + c] * scale;
      }
  }
}

// mode 0: out = v (fp32); 1: out += v (fp32); 2: out = T(float(out) + float(T(v))) (16-bit out,
// the adapter delta rounded to the dtype and added as the reference adds it to its projection).
// A thread owns 4 consecutive columns (N % 4 == 0) for the tile's rows: vector loads and stores.
__device__ __forceinline__ void up_add4_impl(float4& c, const float (&v)[4]) {
  c.x += v[0];
  c.y += v[1];
  c.z += v[2];
  c.w += v[3];
}
template <typename TO>
__device__ __forceinline__ void up_add4_impl(uint2& c, const float (&v)[4]) {
  TO* e = reinterpret_cast<TO*>(&c);
#pragma unroll
  for (int i = 0; i < 4; ++i) e[i] = from_f32<TO>(to_f32(e[i]) + to_f32(from_f32<TO>(v[i])));
}
template <typename TO, typename V>
__device__ __forceinline__ void up_add4(V& c, const float (&v)[4]) {
  if constexpr (sizeof(TO) == 4) up_add4_impl(c, v);
  else up_add4_impl<TO>(c, v);
}

template <typename TO>
__global__ void __launch_bounds__(256) rank_up_kernel(const float* __restrict__ Y, int rk, const float* __restrict__ M,
                                                      int64_t sE, int64_t sj, int64_t sn, int N,
                                                      const int* __restrict__ tiles, float scale, int mode,
                                                      TO* __restrict__ out, int ldo) {
  __shared__ float ys[kTileR][kRk];
  const int e = tiles[blockIdx.x * 3], row0 = tiles[blockIdx.x * 3 + 1], nrows = tiles[blockIdx.x * 3 + 2];
  for (int i = threadIdx.x; i < kTileR * kRk; i += blockDim.x) {
    const int rr = i / kRk, j = i - rr * kRk;
    ys[rr][j] = (rr < nrows && j < rk) ? Y[(int64_t)(row0 + rr) * rk + j] : 0.f;
  }
  __syncthreads();
  const int n0 = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (n0 >= N) return;
  float m[4][kRk];
  const float* Mb = M + (int64_t)e * sE + (int64_t)n0 * sn;
  if (sn == 1 && (sj & 3) == 0 && ((uintptr_t)Mb & 15) == 0) {  // the 4 columns of a rank slot: one vector
#pragma unroll
    for (int j = 0; j < kRk; ++j) {
      const float4 v = j < rk ? *reinterpret_cast<const float4*>(Mb + j * sj) : make_float4(0.f, 0.f, 0.f, 0.f);
      m[0][j] = v.x;
      m[1][j] = v.y;
      m[2][j] = v.z;
      m[3][j] = v.w;
    }
  } else if (sj == 1 && (rk & 3) == 0 && (sn & 3) == 0 && ((uintptr_t)Mb & 15) == 0) {  // a column's rank slots
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int j4 = 0; j4 < kRk; j4 += 4) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j4 < rk) v = *reinterpret_cast<const float4*>(Mb + (int64_t)c * sn + j4);  // rk % 4 == 0 here
        m[c][j4] = v.x;
        m[c][j4 + 1] = v.y;
        m[c][j4 + 2] = v.z;
        m[c][j4 + 3] = v.w;
      }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int j = 0; j < kRk; ++j) m[c][j] = j < rk ? Mb[j * sj + (int64_t)c * sn] : 0.f;
  }
  // rows in batches of 8: the batch's read-modify-writes are in flight together
  using V = typename std::conditional<sizeof(TO) == 4, float4, uint2>::type;
  for (int r0 = 0; r0 < nrows; r0 += 8) {
    V cur[8];
#pragma unroll
    for (int b = 0; b < 8; ++b)
      if (r0 + b < nrows && mode != 0) cur[b] = *reinterpret_cast<const V*>(out + (int64_t)(row0 + r0 + b) * ldo + n0);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (r0 + b >= nrows) break;
      float v[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < kRk; ++j) a = fmaf(ys[r0 + b][j], m[c][j], a);
        v[c] = a * scale;
      }
      if (mode == 0) {
        float4 z = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(out + (int64_t)(row0 + r0 + b) * ldo + n0) = z;
      } else {
        up_add4<TO, V>(cur[b], v);
        *reinterpret_cast<V*>(out + (int64_t)(row0 + r0 + b) * ldo + n0) = cur[b];
      }
    }
  }
}

template <typename TP>
__global__ void __launch_bounds__(256) outer_kernel(const TP* __restrict__ P, int ldp, int A, const float* __restrict__ Y,
                                                    int rk, const int* __restrict__ segs, float scale,
                                                    float* __restrict__ G, int64_t gE, int64_t ga, int64_t gj) {
  __shared__ __align__(16) float ys[kTileR][kRk];
  const int e = segs[blockIdx.x * 3], row0 = segs[blockIdx.x * 3 + 1], nrows = segs[blockIdx.x * 3 + 2];
  const int a = blockIdx.y * blockDim.x + threadIdx.x;
  float acc[kRk];
#pragma unroll
  for (int j = 0; j < kRk; ++j) acc[j] = 0.f;
  for (int r0 = 0; r0 < nrows; r0 += kTileR) {
    __syncthreads();
    for (int i = threadIdx.x; i < kTileR * kRk; i += blockDim.x) {
      const int rr = i / kRk, j = i - rr * kRk;
      ys[rr][j] = (r0 + rr < nrows && j < rk) ? Y[(int64_t)(row0 + r0 + rr) * rk + j] : 0.f;
    }
    __syncthreads();
    if (a < A) {
      const int lim = min(kTileR, nrows - r0);
#pragma unroll 4
      for (int rr = 0; rr < lim; ++rr) {
        const float p = to_f32(P[(int64_t)(row0 + r0 + rr) * ldp + a]);
        const float4* y4 = reinterpret_cast<const float4*>(ys[rr]);
#pragma unroll
        for (int q = 0; q < kRk / 4; ++q) {
          const float4 y = y4[q];
          acc[4 * q] = fmaf(p, y.x, acc[4 * q]);
          acc[4 * q + 1] = fmaf(p, y.y, acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(p, y.z, acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(p, y.w, acc[4 * q + 3]);
        }
      }
    }
  }
  if (a < A)
#pragma unroll
    for (int j = 0; j < kRk; ++j)
      if (j < rk) G[(int64_t)e * gE + (int64_t)a * ga + (int64_t)j * gj] = acc[j] * scale;
}

// bf16 P on the tensor cores: G[a][j] = sum over the segment's rows r of P[r][a] * Y[r][j], with Y
// (fp32) split into three bf16 parts per chunk (as rank_down_mma_kernel splits M). A CTA of four
// warps owns 64 columns a (16 per warp, the M = 16 of an m16n8k16 tile) and all 16 rank slots;
// 32-row chunks of P arrive by cp.async (double-buffered), the A fragments (P transposed) come
// from ldmatrix .trans, and Y's parts are stored transposed so the B fragments are 32-bit loads.
constexpr int kOc = 32;      // rows per chunk
constexpr int kOa = 64;      // columns per CTA
constexpr int kOap = kOa + 8;
constexpr int kOrp = kOc + 8;

__global__ void __launch_bounds__(128) outer_mma_kernel(const __nv_bfloat16* __restrict__ P, int ldp, int A,
                                                        const float* __restrict__ Y, int rk,
                                                        const int* __restrict__ segs, float scale,
                                                        float* __restrict__ G, int64_t gE, int64_t ga, int64_t gj) {
  __shared__ __align__(16) __nv_bfloat16 ps[2][kOc][kOap];
  __shared__ __align__(16) __nv_bfloat16 yt[2][3][kRk][kOrp];
  const int e = segs[blockIdx.x * 3], row0 = segs[blockIdx.x * 3 + 1], nrows = segs[blockIdx.x * 3 + 2];
  const int a0 = blockIdx.y * kOa;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  float yr[kOc * kRk / 128];
  auto issue_p = [&](int r0, int buf) {
#pragma unroll
    for (int u = 0; u < kOc * (kOa / 8) / 128; ++u) {
      const int i = threadIdx.x + 128 * u, rr = i / (kOa / 8), c = (i % (kOa / 8)) * 8;
      const bool ok = r0 + rr < nrows;
      cp_async16(&ps[buf][rr][c], ok ? P + (int64_t)(row0 + r0 + rr) * ldp + a0 + c : P, ok ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto load_y = [&](int r0) {
#pragma unroll
    for (int u = 0; u < kOc * kRk / 128; ++u) {
      const int i = threadIdx.x + 128 * u, rr = i / kRk, j = i % kRk;
      yr[u] = (r0 + rr < nrows && j < rk) ? Y[(int64_t)(row0 + r0 + rr) * rk + j] : 0.f;
    }
  };
  auto store_y = [&](int buf) {
#pragma unroll
    for (int u = 0; u < kOc * kRk / 128; ++u) {
      const int i = threadIdx.x + 128 * u, rr = i / kRk, j = i % kRk;
      const float v = yr[u];
      const __nv_bfloat16 hi = __float2bfloat16_rn(v);
      const float r1 = v - __bfloat162float(hi);
      const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
      yt[buf][0][j][rr] = hi;
      yt[buf][1][j][rr] = mid;
      yt[buf][2][j][rr] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    }
  };
  float acc[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
  issue_p(0, 0);
  load_y(0);
  store_y(0);
  for (int r0 = 0, buf = 0; r0 < nrows; r0 += kOc, buf ^= 1) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    const bool more = r0 + kOc < nrows;
    if (more) {
      issue_p(r0 + kOc, buf ^ 1);
      load_y(r0 + kOc);
    }
#pragma unroll
    for (int ks = 0; ks < kOc; ks += 16) {
      // A (16 columns a x 16 rows r) = P^T: matrix i of the x4 load is rows ks + 8 (i >> 1) .. + 7,
      // columns warp * 16 + 8 (i & 1) .. + 7 of the staged chunk
      const int mi = lane >> 3;
      const uint32_t addr = (uint32_t)__cvta_generic_to_shared(
          &ps[buf][ks + 8 * (mi >> 1) + (lane & 7)][warp * 16 + 8 * (mi & 1)]);
      uint32_t f0, f1, f2, f3;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                   : "=r"(f0), "=r"(f1), "=r"(f2), "=r"(f3)
                   : "r"(addr));
#pragma unroll
      for (int p = 2; p >= 0; --p)
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&yt[buf][p][n * 8 + g][ks + 2 * q]);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&yt[buf][p][n * 8 + g][ks + 2 * q + 8]);
          mma_bf16(acc[n], f0, f1, f2, f3, b0, b1);
        }
    }
    if (more) store_y(buf ^ 1);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int a = a0 + warp * 16 + g + 8 * h;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int j = n * 8 + 2 * q + c;
        if (j < rk && a < A) G[(int64_t)e * gE + (int64_t)a * ga + (int64_t)j * gj] = acc[n][2 * h + c] * scale;
      }
  }
}

}  // namespace
}  // namespace e4b

using namespace e4b;

extern "C" e4b_status e4b_lora_rank_down(const void* X, int x_dtype, int ldx, const float* M, int64_t sE, int64_t sj,
                                         int64_t sk, int rk, int K, const int32_t* tiles, int ntiles, float scale,
                                         float* Y, void* stream) {
  if (rk < 1 || rk > kRk || K < 1 || ntiles < 0) return E4B_ERR_INVALID_ARG;
  if (ntiles == 0) return E4B_OK;
  if (!X || !M || !tiles || !Y) return E4B_ERR_INVALID_ARG;
  if (K % 8 || ldx % 8 || !aligned16(X)) return E4B_ERR_UNSUPPORTED;  // 8-element row loads
  cudaStream_t s = (cudaStream_t)stream;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {  // above 48 KB of shared memory (per process; the attribute is per function)
    cudaError_t a = cudaFuncSetAttribute(rank_down_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         rank_down_smem<__nv_bfloat16>());
    cudaError_t b = cudaFuncSetAttribute(rank_down_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         rank_down_smem<__half>());
    cudaError_t c = cudaFuncSetAttribute(rank_down_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         rank_down_smem<float>());
    attr_err = a != cudaSuccess ? a : b != cudaSuccess ? b : c;
  });
  if (attr_err != cudaSuccess) return E4B_ERR_CUDA;
  // bf16 rows: the tensor-core kernel (E4B_RANK_DOWN_MMA=0: the fp32 CUDA-core kernel)
  static const bool use_mma = [] {
    const char* v = getenv("E4B_RANK_DOWN_MMA");
    return !(v && v[0] == '0');
  }();
  if (x_dtype == E4B_BF16 && use_mma) {
    rank_down_mma_kernel<<<ntiles, 64, 0, s>>>((const __nv_bfloat16*)X, ldx, M, sE, sj, sk, rk, K, tiles, scale, Y);
    return launch_status();
  }
  switch (x_dtype) {
    case E4B_BF16:
      rank_down_kernel<__nv_bfloat16><<<ntiles, 256, rank_down_smem<__nv_bfloat16>(), s>>>(
          (const __nv_bfloat16*)X, ldx, M, sE, sj, sk, rk, K, tiles, scale, Y);
      break;
    case E4B_F16:
      rank_down_kernel<__half><<<ntiles, 256, rank_down_smem<__half>(), s>>>((const __half*)X, ldx, M, sE, sj, sk, rk,
                                                                            K, tiles, scale, Y);
      break;
    case E4B_F32:
      rank_down_kernel<float><<<ntiles, 256, rank_down_smem<float>(), s>>>((const float*)X, ldx, M, sE, sj, sk, rk, K,
                                                                          tiles, scale, Y);
      break;
    default: return E4B_ERR_UNSUPPORTED;
  }
  return launch_status();
}

extern "C" e4b_status e4b_lora_rank_up(const float* Y, int rk, const float* M, int64_t sE, int64_t sj, int64_t sn, int N,
                                       const int32_t* tiles, int ntiles, float scale, int mode, void* out,
                                       int out_dtype, int ldo, void* stream) {
  if (rk < 1 || rk > kRk || N < 1 || ntiles < 0 || mode < 0 || mode > 2) return E4B_ERR_INVALID_ARG;
  if (ntiles == 0) return E4B_OK;
  if (!Y || !M || !tiles || !out) return E4B_ERR_INVALID_ARG;
  if ((mode == 2) != (out_dtype != E4B_F32) || N % 4 || ldo % 4) return E4B_ERR_UNSUPPORTED;
  cudaStream_t s = (cudaStream_t)stream;
  const dim3 grid(ntiles, (N / 4 + 255) / 256);
  switch (out_dtype) {
    case E4B_F32:
      rank_up_kernel<float><<<grid, 256, 0, s>>>(Y, rk, M, sE, sj, sn, N, tiles, scale, mode, (float*)out, ldo);
      break;
    case E4B_BF16:
      rank_up_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(Y, rk, M, sE, sj, sn, N, tiles, scale, mode,
                                                         (__nv_bfloat16*)out, ldo);
      break;
    case E4B_F16:
      rank_up_kernel<__half><<<grid, 256, 0, s>>>(Y, rk, M, sE, sj, sn, N, tiles, scale, mode, (__half*)out, ldo);
      break;
    default: return E4B_ERR_UNSUPPORTED;
  }
  return launch_status();
}

extern "C" e4b_status e4b_lora_outer(const void* P, int p_dtype, int ldp, int A, const float* Y, int rk,
                                     const int32_t* segs, int nsegs, float scale, float* G, int64_t gE, int64_t ga,
                                     int64_t gj, void* stream) {
  if (rk < 1 || rk > kRk || A < 1 || nsegs < 0) return E4B_ERR_INVALID_ARG;
  if (nsegs == 0) return E4B_OK;
  if (!P || !Y || !segs || !G) return E4B_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  // bf16 P with 64-column blocks and 16-byte rows: the tensor-core kernel (E4B_OUTER_MMA=0: CUDA cores)
  static const bool use_mma = [] {
    const char* v = getenv("E4B_OUTER_MMA");
    return !(v && v[0] == '0');
  }();
  if (p_dtype == E4B_BF16 && use_mma && A % kOa == 0 && ldp % 8 == 0 && aligned16(P)) {
    outer_mma_kernel<<<dim3(nsegs, A / kOa), 128, 0, s>>>((const __nv_bfloat16*)P, ldp, A, Y, rk, segs, scale, G, gE,
                                                          ga, gj);
    return launch_status();
  }
  const dim3 grid(nsegs, (A + 255) / 256);
  switch (p_dtype) {
    case E4B_BF16:
      outer_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)P, ldp, A, Y, rk, segs, scale, G, gE, ga,
                                                       gj);
      break;
    case E4B_F16:
      outer_kernel<__half><<<grid, 256, 0, s>>>((const __half*)P, ldp, A, Y, rk, segs, scale, G, gE, ga, gj);
      break;
    case E4B_F32:
      outer_kernel<float><<<grid, 256, 0, s>>>((const float*)P, ldp, A, Y, rk, segs, scale, G, gE, ga, gj);
      break;
    default: return E4B_ERR_UNSUPPORTED;
  }
  return launch_status();
}
