// Router building blocks shared by the router kernels (router.cu) and the fused
// decode step (decode_layer.cu): the fixed-order fp32 logits of one expert and the
// top-k rule of experts4bit_qlora/engines/cpu_router.py:100-119.
#pragma once
#include "common.cuh"

namespace e4b {

constexpr int kRouterTT = 4;      // tokens per CTA

template <int N>
__device__ __forceinline__ void load8_f32(const void* p, int dtype, int64_t i, float (&v)[N]) {
  // loads 8 consecutive elements starting at element i (16- or 32-byte aligned)
  if (dtype == E4B_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 r = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (dtype == E4B_BF16) {
        v[2 * j] = __uint_as_float(w[j] << 16);
        v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      } else {
        __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
        float2 f = __half22float2(h);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    }
  }
}

// One warp: logits of expert e for tokens t0 .. t0 + kRouterTT - 1 (fp32, fixed reduction order:
// lanes accumulate their 8-element slices of 256-element strips in order, then a xor-shuffle sum).
__device__ __forceinline__ void router_logits_warp(const void* __restrict__ x, int x_dtype, const void* __restrict__ wr,
                                                   int w_dtype, int T, int H, int E, int e, int t0,
                                                   float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  float acc[kRouterTT];
#pragma unroll
  for (int j = 0; j < kRouterTT; ++j) acc[j] = 0.f;
  for (int h0 = 0; h0 < H; h0 += 256 * 4) {  // four 256-element strips per lane in flight
    float wv[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int h = h0 + u * 256 + lane * 8;
      if (h < H) load8_f32(wr, w_dtype, (int64_t)e * H + h, wv[u]);
    }
#pragma unroll
    for (int j = 0; j < kRouterTT; ++j) {
      if (t0 + j < T) {
        float xv[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int h = h0 + u * 256 + lane * 8;
          if (h < H) load8_f32(x, x_dtype, (int64_t)(t0 + j) * H + h, xv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (h0 + u * 256 + lane * 8 < H) {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[u][i], wv[u][i], acc[j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kRouterTT; ++j) {
    float a = acc[j];
#pragma unroll
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0 && t0 + j < T) logits[(int64_t)(t0 + j) * E + e] = a;
  }
}

// Eight 16-bit elements (bf16 or fp16) of a raw 16-byte word -> fp32.
__device__ __forceinline__ void unpack8_f32(const uint4& r, int dtype, float (&v)[8]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (dtype == E4B_BF16) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// router_logits_warp with S strips per lane in flight as raw 16-byte words (16-bit x and W_r
// only): the same per-lane accumulation order (strips ascending, elements ascending), so the
// same logits bit for bit; more loads in flight for the latency-bound decode case.
template <int S>
__device__ __forceinline__ void router_logits_warp16(const void* __restrict__ x, int x_dtype,
                                                     const void* __restrict__ wr, int w_dtype, int T, int H, int E,
                                                     int e, int t0, float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  float acc[kRouterTT];
#pragma unroll
  for (int j = 0; j < kRouterTT; ++j) acc[j] = 0.f;
  const uint16_t* wrow = reinterpret_cast<const uint16_t*>(wr) + (int64_t)e * H;
  for (int h0 = 0; h0 < H; h0 += 256 * S) {
    uint4 wraw[S];
#pragma unroll
    for (int u = 0; u < S; ++u) {
      const int h = h0 + u * 256 + lane * 8;
      wraw[u] = h < H ? *reinterpret_cast<const uint4*>(wrow + h) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kRouterTT; ++j) {
      if (t0 + j < T) {
        const uint16_t* xrow = reinterpret_cast<const uint16_t*>(x) + (int64_t)(t0 + j) * H;
        uint4 xraw[S];
#pragma unroll
        for (int u = 0; u < S; ++u) {
          const int h = h0 + u * 256 + lane * 8;
          xraw[u] = h < H ? *reinterpret_cast<const uint4*>(xrow + h) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < S; ++u) {
          if (h0 + u * 256 + lane * 8 < H) {
            float xv[8], wv[8];
            unpack8_f32(xraw[u], x_dtype, xv);
            unpack8_f32(wraw[u], w_dtype, wv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[j] = fmaf(xv[i], wv[i], acc[j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kRouterTT; ++j) {
    float a = acc[j];
#pragma unroll
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0 && t0 + j < T) logits[(int64_t)(t0 + j) * E + e] = a;
  }
}

// One warp, token t: the sum of the logit slices (fixed order), softmax / top-k / renorm as
// cpu_router.route_on_host. Lane j < k receives the j-th selection (expert, weight).
template <int EPL>
__device__ __forceinline__ void router_topk_warp(const float* __restrict__ logits, int nsplit,
                                                 float* __restrict__ logits_sum, int T, int E, int k, int kind,
                                                 int renorm, int t, int& out_e, float& out_w) {
  const int lane = threadIdx.x & 31;
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = -INFINITY;
    if (e < E) {
      float acc = logits[(int64_t)t * E + e];
      for (int z = 1; z < nsplit; ++z) acc += logits[((int64_t)z * T + t) * E + e];  // fixed slice order
      if (logits_sum) logits_sum[(int64_t)t * E + e] = acc;
      v[i] = acc;
    }
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float denom = 0.f;
  if (kind == E4B_SOFTMAX_THEN_TOPK) {
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i < E) denom += expf(v[i] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, o);
  }
  uint32_t taken = 0;
  float sel_v = 0.f;   // lane j (< k) keeps the j-th selection
  int sel_e = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(taken >> i & 1u) && (v[i] > bv || be == 0x7fffffff)) {
        bv = v[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if ((be & 31) == lane && be < E) taken |= 1u << (be >> 5);
    if (lane == j) {
      sel_v = bv;
      sel_e = be;
    }
  }
  float w;
  if (kind == E4B_SOFTMAX_THEN_TOPK) {
    w = expf(sel_v - m) / denom;
  } else {
    // softmax over the k selected logits; the first selection is their max
    const float top = __shfl_sync(0xffffffffu, sel_v, 0);
    w = expf(sel_v - top);
  }
  float s = 0.f;
  const bool need_sum = (kind == E4B_TOPK_THEN_SOFTMAX) || renorm;
  if (need_sum) {
    // fixed-order sum over the k selections (slot order)
    for (int j = 0; j < k; ++j) s += __shfl_sync(0xffffffffu, w, j);
    w = w / s;
  }
  out_e = sel_e;
  out_w = w;
}


// The iterative selection as a call, not inlined (the rare path of the ranked version).
template <int EPL>
__device__ __noinline__ void router_topk_warp_outlined(const float* logits, int T, int E, int k, int kind, int renorm,
                                                       int t, int& out_e, float& out_w) {
  router_topk_warp<EPL>(logits, 1, nullptr, T, E, k, kind, renorm, t, out_e, out_w);
}

// router_topk_warp for logits already in shared memory (nsplit = 1): each lane ranks its
// values against all E logits (descending, ties to the lower id) instead of k rounds of
// warp-wide argmax, and the selections are scattered to their slots through sel_v / sel_e
// (shared, k entries per warp). The same selections and the same weight arithmetic as
// router_topk_warp; a NaN logit anywhere falls back to it.
template <int EPL>
__device__ __forceinline__ void router_topk_warp_ranked(const float* __restrict__ logits, int T, int E, int k,
                                                        int kind, int renorm, int t, float* sel_vs, int* sel_es,
                                                        int& out_e, float& out_w) {
  const int lane = threadIdx.x & 31;
  const float* row = logits + (int64_t)t * E;
  float v[EPL];
  bool nan = false;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? row[e] : -INFINITY;
    nan |= isnan(v[i]);
  }
  if (__any_sync(0xffffffffu, nan)) {
    router_topk_warp_outlined<EPL>(logits, T, E, k, kind, renorm, t, out_e, out_w);
    return;
  }
  int rank[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) rank[i] = 0;
  for (int e2 = 0; e2 < E; ++e2) {
    const float o = row[e2];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      rank[i] += (o > v[i]) || (o == v[i] && e2 < e);
    }
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E && rank[i] < k) {
      sel_vs[rank[i]] = v[i];
      sel_es[rank[i]] = e;
    }
  }
  __syncwarp();
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float denom = 0.f;
  if (kind == E4B_SOFTMAX_THEN_TOPK) {
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i < E) denom += expf(v[i] - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, o);
  }
  const float sel_v = lane < k ? sel_vs[lane] : 0.f;
  const int sel_e = lane < k ? sel_es[lane] : 0;
  __syncwarp();
  float w;
  if (kind == E4B_SOFTMAX_THEN_TOPK) {
    w = expf(sel_v - m) / denom;
  } else {
    const float top = __shfl_sync(0xffffffffu, sel_v, 0);
    w = expf(sel_v - top);
  }
  float s = 0.f;
  const bool need_sum = (kind == E4B_TOPK_THEN_SOFTMAX) || renorm;
  if (need_sum) {
    for (int j = 0; j < k; ++j) s += __shfl_sync(0xffffffffu, w, j);
    w = w / s;
  }
  out_e = sel_e;
  out_w = w;
}

}  // namespace e4b
