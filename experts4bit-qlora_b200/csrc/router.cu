// Router (R1): fp32 logits x . W_r^T, then top-k with the rule of
// experts4bit_qlora/engines/cpu_router.py:100-119 -- stable descending order,
// ties to the LOWER expert id -- and the routing epilogue of route_on_host
// (softmax over all logits then select [+ renorm], or select then softmax).
#include "common.cuh"

namespace e4b {

constexpr int kRouterWarps = 8;   // experts per CTA (one warp each)
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

__global__ void __launch_bounds__(kRouterWarps * 32)
router_logits_kernel(const void* __restrict__ x, int x_dtype, const void* __restrict__ wr, int w_dtype, int T, int H,
                     int E, float* __restrict__ logits) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouterWarps + warp;
  const int t0 = blockIdx.y * kRouterTT;
  if (e >= E) return;
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

// One warp per token; EPL = experts per lane (E <= 32 * EPL).
template <int EPL>
__global__ void router_topk_kernel(const float* __restrict__ logits, int T, int E, int k, int kind, int renorm,
                                   int64_t* __restrict__ topk_idx, float* __restrict__ topk_w) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? logits[(int64_t)t * E + e] : -INFINITY;
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
  if (lane < k) {
    topk_idx[(int64_t)t * k + lane] = sel_e;
    topk_w[(int64_t)t * k + lane] = w;
  }
}

}  // namespace e4b

using namespace e4b;

extern "C" size_t e4b_router_workspace_bytes(int T, int E) {
  if (T < 0 || E < 0) return 0;
  return kErrBytes + align_up((size_t)T * E * sizeof(float), 256);
}

extern "C" e4b_status e4b_router_topk(const void* x, int x_dtype, const void* w_router, int w_dtype, int T, int H,
                                      int E, int k, int kind, int norm_topk_prob, float* logits_out,
                                      int64_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (T < 0 || H <= 0 || E <= 0 || k <= 0 || k > E || k > 32 || E > 1024) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(x_dtype) || !is_any_dtype(w_dtype) || H % 8) return E4B_ERR_UNSUPPORTED;
  if (kind != E4B_SOFTMAX_THEN_TOPK && kind != E4B_TOPK_THEN_SOFTMAX) return E4B_ERR_INVALID_ARG;
  if (T == 0) return E4B_OK;
  if (!x || !w_router || !topk_idx || !topk_w) return E4B_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_router)) return E4B_ERR_ALIGNMENT;
  float* logits = logits_out;
  if (!logits) {
    if (!workspace || workspace_bytes < e4b_router_workspace_bytes(T, E)) return E4B_ERR_WORKSPACE;
    logits = reinterpret_cast<float*>(static_cast<char*>(workspace) + kErrBytes);
  }
  cudaStream_t s = (cudaStream_t)stream;
  dim3 g1((E + kRouterWarps - 1) / kRouterWarps, (T + kRouterTT - 1) / kRouterTT);
  router_logits_kernel<<<g1, kRouterWarps * 32, 0, s>>>(x, x_dtype, w_router, w_dtype, T, H, E, logits);
  const int warps = 8;
  const int g2 = (T + warps - 1) / warps;
  if (E <= 32)
    router_topk_kernel<1><<<g2, warps * 32, 0, s>>>(logits, T, E, k, kind, norm_topk_prob, topk_idx, topk_w);
  else if (E <= 64)
    router_topk_kernel<2><<<g2, warps * 32, 0, s>>>(logits, T, E, k, kind, norm_topk_prob, topk_idx, topk_w);
  else if (E <= 128)
    router_topk_kernel<4><<<g2, warps * 32, 0, s>>>(logits, T, E, k, kind, norm_topk_prob, topk_idx, topk_w);
  else if (E <= 256)
    router_topk_kernel<8><<<g2, warps * 32, 0, s>>>(logits, T, E, k, kind, norm_topk_prob, topk_idx, topk_w);
  else
    router_topk_kernel<32><<<g2, warps * 32, 0, s>>>(logits, T, E, k, kind, norm_topk_prob, topk_idx, topk_w);
  return launch_status();
}
