// Router (R1): fp32 logits x . W_r^T, then top-k with the rule of
// experts4bit_qlora/engines/cpu_router.py:100-119 -- stable descending order,
// ties to the LOWER expert id -- and the routing epilogue of route_on_host
// (softmax over all logits then select [+ renorm], or select then softmax).
#include <type_traits>

#include "common.cuh"
#include "router.cuh"

namespace e4b {

constexpr int kRouterWarps = 8;   // experts per CTA (one warp each)

template <typename T> __device__ __forceinline__ void mma_act(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                              uint32_t a3, uint32_t b0, uint32_t b1);
template <> __device__ __forceinline__ void mma_act<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                                   uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <> __device__ __forceinline__ void mma_act<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                            uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__global__ void __launch_bounds__(kRouterWarps * 32)
router_logits_kernel(const void* __restrict__ x, int x_dtype, const void* __restrict__ wr, int w_dtype, int T, int H,
                     int E, float* __restrict__ logits) {
  const int e = blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (e >= E) return;
  router_logits_warp(x, x_dtype, wr, w_dtype, T, H, E, e, blockIdx.y * kRouterTT, logits);
}

// Many tokens: logits as a tensor-core GEMM. A CTA takes 64 tokens x 64 experts over
// one K slice of `ks_len` elements (blockIdx.z); its 4 warps each own 16 tokens x 64
// experts (n8 tiles of mma.sync m16n8k16, bf16 or fp16 operands, fp32 accumulation;
// tiles past E are skipped). 64-wide K chunks of x and W_r are staged in padded
// shared memory (weights of another type are rounded to the activation type there).
// Slice z writes its partial logits to logits + z*T*E; the top-k kernel sums the
// slices in order, so the result does not depend on scheduling.
template <typename T>
__device__ __forceinline__ uint4 load8_as(const void* p, int dtype, int64_t i) {
  if (dtype == (sizeof(T) == 2 && std::is_same<T, __half>::value ? E4B_F16 : E4B_BF16))
    return *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(p) + i * 2);
  float v[8];
  if (dtype == E4B_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = load_as_f32(p, dtype, i + j);
  }
  return make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
}

template <typename T>
__global__ void __launch_bounds__(128) router_logits_mma_kernel(const T* __restrict__ x, const void* __restrict__ wr,
                                                                int w_dtype, int Tn, int H, int E, int ks_len,
                                                                float* __restrict__ logits) {
  constexpr int P = 72;  // padded row, halves
  __shared__ __align__(16) T xs[64][P];
  __shared__ __align__(16) T ws[64][P];
  const int t0 = blockIdx.x * 64, e0 = blockIdx.y * 64;
  const int kb = blockIdx.z * ks_len, ke = min(H, kb + ks_len);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, q = lane & 3;
  const int ntiles = min(8, (E - e0 + 7) / 8);
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
  for (int k0 = kb; k0 < ke; k0 += 64) {
    for (int i = threadIdx.x; i < 64 * 8; i += 128) {
      const int rr = i >> 3, v = i & 7;
      uint4 xv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
      if (t0 + rr < Tn) xv = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + rr) * H + k0 + v * 8);
      if (e0 + rr < E) wv = load8_as<T>(wr, w_dtype, (int64_t)(e0 + rr) * H + k0 + v * 8);
      *reinterpret_cast<uint4*>(&xs[rr][v * 8]) = xv;
      *reinterpret_cast<uint4*>(&ws[rr][v * 8]) = wv;
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < 64; ks += 16) {
      const int rw = warp * 16 + gq;
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&xs[rw][ks + 2 * q]);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(&xs[rw + 8][ks + 2 * q]);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&xs[rw][ks + 2 * q + 8]);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(&xs[rw + 8][ks + 2 * q + 8]);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < ntiles) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&ws[n * 8 + gq][ks + 2 * q]);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&ws[n * 8 + gq][ks + 2 * q + 8]);
          mma_act<T>(acc[n], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    __syncthreads();
  }
  float* out = logits + (int64_t)blockIdx.z * Tn * E;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int t = t0 + warp * 16 + gq + 8 * h;
    if (t >= Tn) continue;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int e = e0 + n * 8 + 2 * q + c;
        if (e < E) out[(int64_t)t * E + e] = acc[n][2 * h + c];
      }
  }
}

// K slices of the tensor-core logits: enough CTAs to cover the SMs twice, each slice
// a multiple of 64 elements.
inline int router_ks_len(int T, int H, int E) {
  const int ctas = ((T + 63) / 64) * ((E + 63) / 64);
  const int chunks = H / 64;
  int splits = (296 + ctas - 1) / ctas;
  splits = splits < 1 ? 1 : (splits > 16 ? 16 : splits);
  if (splits > chunks) splits = chunks;
  return ((chunks + splits - 1) / splits) * 64;
}
inline bool router_uses_mma(int T, int H) { return T > 16 && H % 64 == 0; }

// One warp per token; EPL = experts per lane (E <= 32 * EPL).
template <int EPL>
__global__ void router_topk_kernel(const float* __restrict__ logits, int nsplit, float* __restrict__ logits_sum,
                                   int T, int E, int k, int kind, int renorm, int64_t* __restrict__ topk_idx,
                                   float* __restrict__ topk_w) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  int sel_e;
  float w;
  router_topk_warp<EPL>(logits, nsplit, logits_sum, T, E, k, kind, renorm, t, sel_e, w);
  const int lane = threadIdx.x & 31;
  if (lane < k) {
    topk_idx[(int64_t)t * k + lane] = sel_e;
    topk_w[(int64_t)t * k + lane] = w;
  }
}

}  // namespace e4b

using namespace e4b;

extern "C" size_t e4b_router_workspace_bytes(int T, int E) {
  if (T < 0 || E < 0) return 0;
  // room for the largest K split (16 slices of partial logits)
  return kErrBytes + align_up((size_t)T * E * sizeof(float) * 16, 256);
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
  cudaStream_t s = (cudaStream_t)stream;
  const bool mma = router_uses_mma(T, H);
  const int ks_len = mma ? router_ks_len(T, H, E) : H;
  const int nsplit = (H + ks_len - 1) / ks_len;
  float* logits = logits_out;
  float* logits_sum = nullptr;
  if (!logits || nsplit > 1) {
    if (!workspace || workspace_bytes < e4b_router_workspace_bytes(T, E)) return E4B_ERR_WORKSPACE;
    logits = reinterpret_cast<float*>(static_cast<char*>(workspace) + kErrBytes);
    logits_sum = logits_out;  // the summed slices, when the caller wants the logits
  }
  if (mma) {
    dim3 g1((T + 63) / 64, (E + 63) / 64, nsplit);
    if (x_dtype == E4B_BF16)
      router_logits_mma_kernel<__nv_bfloat16><<<g1, 128, 0, s>>>((const __nv_bfloat16*)x, w_router, w_dtype, T, H, E,
                                                                 ks_len, logits);
    else
      router_logits_mma_kernel<__half><<<g1, 128, 0, s>>>((const __half*)x, w_router, w_dtype, T, H, E, ks_len,
                                                          logits);
  } else {
    dim3 g1((E + kRouterWarps - 1) / kRouterWarps, (T + kRouterTT - 1) / kRouterTT);
    router_logits_kernel<<<g1, kRouterWarps * 32, 0, s>>>(x, x_dtype, w_router, w_dtype, T, H, E, logits);
  }
  const int warps = 8;
  const int g2 = (T + warps - 1) / warps;
#define E4B_TOPK(EPL) \
  router_topk_kernel<EPL><<<g2, warps * 32, 0, s>>>(logits, nsplit, logits_sum, T, E, k, kind, norm_topk_prob, topk_idx, topk_w)
  if (E <= 32)
    E4B_TOPK(1);
  else if (E <= 64)
    E4B_TOPK(2);
  else if (E <= 128)
    E4B_TOPK(4);
  else if (E <= 256)
    E4B_TOPK(8);
  else
    E4B_TOPK(32);
#undef E4B_TOPK
  return launch_status();
}
