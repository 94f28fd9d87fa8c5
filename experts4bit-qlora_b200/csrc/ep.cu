// Expert parallelism: the layer split at its two exchanges.
//
// Rank p of P owns experts [p*E/P, (p+1)*E/P) (contiguous slices of the packed
// stacks) and a shard of the tokens. One layer is
//   source side   e4b_ep_dispatch: permute the shard's picks by global expert
//                 (the same stable order as the single-GPU layer) and gather
//                 their rows, so the rows bound for each rank are contiguous;
//   exchange      per-expert counts, then the rows (all-to-all, caller's NCCL);
//   expert side   e4b_ep_experts: regroup the received rows (source-major) by
//                 local expert while converting them to fp16, run the expert
//                 stages of the fused layer, and write the down rows back in
//                 the received (source-major) order;
//   exchange      the down rows return on the reverse all-to-all, landing in
//                 the source's sorted order;
//   source side   e4b_combine with the permutation's inverse: the fixed slot
//                 order makes the result independent of P.
// The reference has no distributed code; the split follows the per-expert
// independence of its loop (experts4bit_qlora/_vendor/experts.py:486-513).
#include "moe_stages.cuh"
#include "permute.cuh"
#include "lora.cuh"
#include "umma.cuh"

namespace e4b {

namespace {

// dst[r] = src[map[r]] for 16-bit rows of K elements (K % 8 == 0); block 0 also
// writes counts[e] = offsets[e+1] - offsets[e].
__global__ void __launch_bounds__(256) ep_gather_rows_kernel(const uint4* __restrict__ src,
                                                             const int32_t* __restrict__ map, int R, int vec_per_row,
                                                             uint4* __restrict__ dst,
                                                             const int32_t* __restrict__ offsets, int E,
                                                             int32_t* __restrict__ counts) {
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = offsets[e + 1] - offsets[e];
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < R; r += gridDim.x * 8) {
    const uint4* s = src + (int64_t)map[r] * vec_per_row;
    uint4* d = dst + (int64_t)r * vec_per_row;
    for (int v = lane; v < vec_per_row; v += 32) d[v] = s[v];
  }
}

// dst[map[r]] = src[r] for 16-bit rows.
__global__ void __launch_bounds__(256) ep_scatter_rows_kernel(const uint4* __restrict__ src,
                                                              const int32_t* __restrict__ map, int R, int vec_per_row,
                                                              uint4* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < R; r += gridDim.x * 8) {
    const uint4* s = src + (int64_t)r * vec_per_row;
    uint4* d = dst + (int64_t)map[r] * vec_per_row;
    for (int v = lane; v < vec_per_row; v += 32) d[v] = s[v];
  }
}

struct PlanArgs {
  const int32_t* recv_counts;  // [P, El]: rows source p sent for local expert e
  int P, El, R;
  int32_t* offsets;            // [El+1] expert-major segment starts
  int32_t* active;             // [El]
  int32_t* num_active;
  int32_t* tile_a;             // [El+1] prefix of ceil(count / tile_a_rows)
  int32_t* tile_b;             // [El+1] prefix of ceil(count / tile_b_rows)
  int tile_a_rows, tile_b_rows;
  int32_t* src_start;          // [P*El] source-major start of block (p, e)
  int32_t* dst_start;          // [P*El] expert-major start of block (p, e)
  int32_t* map;                // [R] expert-major row -> source-major row
  int* err;
};

// One CTA: segment tables of the received rows and the expert-major -> source-major
// row map. Received rows are source-major, and within a source expert-major (the
// order the source's permutation produced); the expert stages want expert-major,
// and within an expert source-major. Block starts come from two exclusive scans
// over the P x El count matrix (source-major and expert-major), done with a
// shared-memory scan over chunks of 1024 blocks.
__device__ __forceinline__ int block_scan_exclusive(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) s_warp[lane] = w;
  }
  __syncthreads();
  const int excl = x - v + (warp ? s_warp[warp - 1] : 0);
  total = s_warp[nw - 1];
  __syncthreads();
  return excl;
}

__global__ void __launch_bounds__(1024) ep_plan_kernel(PlanArgs a) {
  __shared__ int s_warp[32];
  __shared__ int s_n;
  const int tid = threadIdx.x;
  const int nb = a.P * a.El;
  // source-major starts: block b = p * El + e in storage order
  int carry = 0;
  for (int b0 = 0; b0 < nb; b0 += blockDim.x) {
    const int b = b0 + tid;
    const int v = b < nb ? max(a.recv_counts[b], 0) : 0;
    int tot;
    const int ex = block_scan_exclusive(v, s_warp, tot);
    if (b < nb) a.src_start[b] = carry + ex;
    carry += tot;
  }
  // expert-major starts: position j = e * P + p
  carry = 0;
  for (int j0 = 0; j0 < nb; j0 += blockDim.x) {
    const int j = j0 + tid;
    const int e = j / a.P, p = j - e * a.P;
    const int v = j < nb ? max(a.recv_counts[p * a.El + e], 0) : 0;
    int tot;
    const int ex = block_scan_exclusive(v, s_warp, tot);
    if (j < nb) a.dst_start[p * a.El + e] = carry + ex;
    carry += tot;
  }
  const int total = carry;
  __syncthreads();  // starts visible to the whole block
  // per-expert segment tables and tile prefixes (scan over experts)
  if (tid == 0) s_n = 0;
  carry = 0;
  int ta_carry = 0, tb_carry = 0;
  for (int e0 = 0; e0 < a.El; e0 += blockDim.x) {
    const int e = e0 + tid;
    int c = 0;
    if (e < a.El)
      for (int p = 0; p < a.P; ++p) c += max(a.recv_counts[p * a.El + e], 0);
    int tot, tta, ttb;
    const int ex = block_scan_exclusive(c, s_warp, tot);
    const int exa = block_scan_exclusive((c + a.tile_a_rows - 1) / a.tile_a_rows, s_warp, tta);
    const int exb = block_scan_exclusive((c + a.tile_b_rows - 1) / a.tile_b_rows, s_warp, ttb);
    if (e < a.El) {
      a.offsets[e] = carry + ex;
      a.tile_a[e] = ta_carry + exa;
      a.tile_b[e] = tb_carry + exb;
    }
    carry += tot;
    ta_carry += tta;
    tb_carry += ttb;
  }
  // active list in ascending order
  for (int e0 = 0; e0 < a.El; e0 += blockDim.x) {
    const int e = e0 + tid;
    int c = 0;
    if (e < a.El)
      for (int p = 0; p < a.P; ++p) c += max(a.recv_counts[p * a.El + e], 0);
    int tot;
    const int ex = block_scan_exclusive(c > 0 ? 1 : 0, s_warp, tot);
    if (e < a.El && c > 0) a.active[s_n + ex] = e;
    __syncthreads();
    if (tid == 0) s_n += tot;
    __syncthreads();
  }
  if (tid == 0) {
    a.offsets[a.El] = total;
    a.tile_a[a.El] = ta_carry;
    a.tile_b[a.El] = tb_carry;
    *a.num_active = s_n;
    if (total != a.R) raise_error(a.err, E4B_ERR_INVALID_ARG);
  }
  __syncthreads();
  // map fill: one warp per (source, expert) block
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  for (int b = warp; b < nb; b += nwarps) {
    const int c = a.recv_counts[b];
    const int s0 = a.src_start[b], d0 = a.dst_start[b];
    for (int i = lane; i < c; i += 32)
      if (d0 + i < a.R && s0 + i < a.R) a.map[d0 + i] = s0 + i;
  }
  // rows no block covers (only when the counts disagree with R) map to row 0
  for (int i = total + tid; i < a.R; i += blockDim.x) a.map[i] = 0;
}

int rows_ctas(int rows) {
  int c = (rows + 7) / 8;
  return c < 1 ? 1 : (c > 148 * 8 ? 148 * 8 : c);
}

struct EpLayout {
  size_t offsets, active, num_active, tile_a, tile_b, src_start, dst_start, map, x16, x_scale, h, down_rows, xa_gu,
      xa_dn, umma, total;
};

EpLayout ep_layout(const e4b_moe_desc& d, int P) {
  EpLayout L{};
  const size_t R = (size_t)d.tokens;
  const size_t E = d.num_experts;
  size_t o = kErrBytes;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.offsets = take((E + 1) * 4);
  L.active = take(E * 4);
  L.num_active = take(4);
  L.tile_a = take((E + 1) * 4);
  L.tile_b = take((E + 1) * 4);
  L.src_start = take((size_t)P * E * 4);
  L.dst_start = take((size_t)P * E * 4);
  L.map = take(R * 4);
  L.x16 = take(R * d.hidden * 2);
  L.x_scale = take(R * 4);
  L.h = take(R * d.intermediate * 2);
  L.down_rows = take(R * d.hidden * 2);
  // LoRA-A products: fp32 [R, rank] for the GEMV path, fp16 [R, 64] for the tensor-core path
  const size_t xa_bytes = d.lora_rank > 0 ? (R * d.lora_rank * 4 > R * 128 ? R * d.lora_rank * 4 : R * 128) : 0;
  L.xa_gu = take(xa_bytes);
  L.xa_dn = take(xa_bytes);
  L.umma = take(umma_workspace_bytes((int)R, 1, d.num_experts, d.hidden, d.intermediate));
  L.total = o;
  return L;
}

bool ep_desc_ok(const e4b_moe_desc& d, int P) {
  if (P <= 0 || P > 1024) return false;
  if (d.num_experts <= 0 || d.num_experts > 1024 || (int64_t)d.num_experts * P > (1 << 20)) return false;
  if (d.hidden <= 0 || d.intermediate <= 0 || d.tokens < 0 || d.tokens > (1 << 30)) return false;
  if (d.top_k != 1) return false;
  return true;
}

}  // namespace

}  // namespace e4b

using namespace e4b;

extern "C" size_t e4b_ep_dispatch_workspace_bytes(int T, int k, int E) {
  if (T < 0 || k <= 0 || E <= 0 || E > 1024) return 0;
  return kErrBytes + align_up((size_t)(E + 1) * 4, 256) + align_up((size_t)T * k * 4, 256);
}

extern "C" e4b_status e4b_ep_dispatch(const void* hidden, int act_dtype, const int64_t* topk_idx, int T, int k, int E,
                                      int H, void* send_rows, int32_t* expert_counts, int32_t* inv, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (T < 0 || k <= 0 || k > 32 || k > E || E <= 0 || E > 1024 || H <= 0 || (int64_t)T * k > (1 << 30))
    return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(act_dtype) || H % 8) return E4B_ERR_UNSUPPORTED;
  if (!expert_counts) return E4B_ERR_INVALID_ARG;
  if (T > 0 && (!hidden || !topk_idx || !send_rows || !inv)) return E4B_ERR_INVALID_ARG;
  if (T > 0 && (!aligned16(hidden) || !aligned16(send_rows))) return E4B_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < e4b_ep_dispatch_workspace_bytes(T, k, E)) return E4B_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + kErrBytes);
  int32_t* sorted_token = reinterpret_cast<int32_t*>(ws + kErrBytes + align_up((size_t)(E + 1) * 4, 256));
  PermuteArgs pa{};
  pa.topk_idx = topk_idx;
  pa.T = T;
  pa.k = k;
  pa.E = E;
  pa.inv = inv;
  pa.sorted_token = sorted_token;
  pa.offsets = offsets;
  pa.tile_a = kLoraRows;
  pa.tile_b = kUmmaTokens;
  pa.err = reinterpret_cast<int*>(ws);
  pa.reset_err = 1;
  e4b_status st = launch_permute(pa, s);
  if (st != E4B_OK) return st;
  const int R = T * k;
  ep_gather_rows_kernel<<<rows_ctas(R), 256, 0, s>>>(static_cast<const uint4*>(hidden), sorted_token, R, H / 8,
                                                     static_cast<uint4*>(send_rows), offsets, E, expert_counts);
  return launch_status();
}

extern "C" size_t e4b_ep_experts_workspace_bytes(const e4b_moe_desc* local, int world) {
  if (!local || !ep_desc_ok(*local, world)) return 0;
  return ep_layout(*local, world).total;
}

extern "C" e4b_status e4b_ep_experts(const e4b_moe_desc* local, int world, const int32_t* recv_counts,
                                     const e4b_moe_tensors* t, void* workspace, size_t workspace_bytes, void* stream) {
  if (!local || !t || !ep_desc_ok(*local, world)) return E4B_ERR_INVALID_ARG;
  const e4b_moe_desc& d = *local;
  if (!is_act_dtype(d.act_dtype) || d.out_dtype != E4B_F16) return E4B_ERR_UNSUPPORTED;
  if (d.hidden % 64 || d.intermediate % 64) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank < 0 || d.lora_rank > kLoraMaxRank) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank > 0 && !is_any_dtype(d.lora_dtype)) return E4B_ERR_UNSUPPORTED;
  if (e4b_status fs = check_weight_format(d)) return fs;
  const int R = d.tokens, El = d.num_experts, H = d.hidden, I = d.intermediate;
  if (!recv_counts || !t->gate_up_packed || !t->gate_up_absmax || !t->down_packed || !t->down_absmax)
    return E4B_ERR_INVALID_ARG;
  if (R > 0 && (!t->hidden || !t->out)) return E4B_ERR_INVALID_ARG;
  if (d.lora_rank > 0 && (!t->gate_up_lora_A || !t->gate_up_lora_B || !t->down_lora_A || !t->down_lora_B))
    return E4B_ERR_INVALID_ARG;
  if (!aligned16(t->gate_up_packed) || !aligned16(t->down_packed)) return E4B_ERR_ALIGNMENT;
  if (R > 0 && (!aligned16(t->hidden) || !aligned16(t->out))) return E4B_ERR_ALIGNMENT;
  const EpLayout L = ep_layout(d, world);
  if (!workspace || workspace_bytes < L.total) return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) return E4B_ERR_CUDA;
  mark_stage(t, 0, s);
  PlanArgs pl{};
  pl.recv_counts = recv_counts;
  pl.P = world;
  pl.El = El;
  pl.R = R;
  pl.offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  pl.active = reinterpret_cast<int32_t*>(ws + L.active);
  pl.num_active = reinterpret_cast<int32_t*>(ws + L.num_active);
  pl.tile_a = reinterpret_cast<int32_t*>(ws + L.tile_a);
  pl.tile_b = reinterpret_cast<int32_t*>(ws + L.tile_b);
  pl.tile_a_rows = kLoraRows;
  pl.tile_b_rows = kUmmaTokens;
  pl.src_start = reinterpret_cast<int32_t*>(ws + L.src_start);
  pl.dst_start = reinterpret_cast<int32_t*>(ws + L.dst_start);
  pl.map = reinterpret_cast<int32_t*>(ws + L.map);
  pl.err = err;
  ep_plan_kernel<<<1, 1024, 0, s>>>(pl);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  if (R == 0) {
    mark_stage(t, 6, s);
    return E4B_OK;
  }
  __half* x16 = reinterpret_cast<__half*>(ws + L.x16);
  float* x_scale = reinterpret_cast<float*>(ws + L.x_scale);
  ConvertArgs cv{};
  cv.src = t->hidden;
  cv.src_dtype = d.act_dtype;
  cv.dst = x16;
  cv.scale = x_scale;
  cv.rows = R;
  cv.K = H;
  e4b_status st = launch_gather_convert(cv, pl.map, s);
  if (st != E4B_OK) return st;
  mark_stage(t, 1, s);

  ExpertRows x{};
  x.x16 = x16;
  x.x_scale = x_scale;
  x.a_rows = nullptr;
  x.x_rows = R;
  x.R = R;
  x.max_rows_per_expert = R;
  x.offsets = pl.offsets;
  x.active = pl.active;
  x.num_active = pl.num_active;
  x.tile_a = pl.tile_a;
  x.tile_b = pl.tile_b;
  // The same regime rule as the single-GPU layer: average rows per local expert.
  x.use_umma = umma_worthwhile(R, El) && umma_eligible(R, 1, El, H, I, d.has_gate, d.act_dtype, d.lora_rank);
  x.h = ws + L.h;
  x.down_rows = ws + L.down_rows;
  x.xa_gu = reinterpret_cast<float*>(ws + L.xa_gu);
  x.xa_dn = reinterpret_cast<float*>(ws + L.xa_dn);
  x.umma_scratch = ws + L.umma;
  x.err = err;
  if ((st = run_expert_stages(d, t, x, s)) != E4B_OK) return st;
  ep_scatter_rows_kernel<<<rows_ctas(R), 256, 0, s>>>(static_cast<const uint4*>(x.down_rows), pl.map, R, H / 8,
                                                      static_cast<uint4*>(t->out));
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  mark_stage(t, 6, s);
  return E4B_OK;
}
