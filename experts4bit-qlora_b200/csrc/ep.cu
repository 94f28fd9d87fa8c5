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
#include <cuda.h>

#include <cstring>

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
  // Peer-memory exchange: source p's rows start at p * src_stride (fixed regions, not packed),
  // and R is a capacity (the counts may sum to less). Both 0 for packed rows.
  int src_stride;
  int partial;
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
  if (a.src_stride > 0) {
    // fixed source regions: restart the prefix at each source, at p * src_stride
    __syncthreads();
    for (int b0 = 0; b0 < nb; b0 += blockDim.x) {
      const int b = b0 + tid;
      int v = 0;
      if (b < nb) {
        const int p = b / a.El, e = b - p * a.El;
        int pre = 0;
        for (int j = 0; j < e; ++j) pre += max(a.recv_counts[p * a.El + j], 0);
        v = p * a.src_stride + pre;
      }
      __syncthreads();
      if (b < nb) a.src_start[b] = v;
    }
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
    if (a.partial ? total > a.R : total != a.R) raise_error(a.err, E4B_ERR_INVALID_ARG);
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
  if (!a.partial)
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
  pa.reset_err = 0;  // the error word is sticky: only e4b_read_device_error clears it
  e4b_status st = launch_permute(pa, s);
  if (st != E4B_OK) return st;
  const int R = T * k;
  ep_gather_rows_kernel<<<rows_ctas(R), 256, 0, s>>>(static_cast<const uint4*>(hidden), sorted_token, R, H / 8,
                                                     static_cast<uint4*>(send_rows), offsets, E, expert_counts);
  return launch_status();
}

// ---- Peer-memory exchange ----------------------------------------------------
namespace e4b {

namespace {

constexpr int kMaxPeers = E4B_EP_MAX_PEERS;
// Bounded waits on a peer's arrival flag: at most this many polls, 256 ns apart (~4 s).
constexpr int kPeerWaitPolls = 1 << 24;

// Offsets inside one rank's exchange region (identical on every rank of a group).
struct PeerLayout {
  size_t recv_flag, ret_flag, done, calls, counts, recv_off, recv_rows, ret_rows, total;
};

PeerLayout peer_layout(int P, int El, int cap, int H) {
  PeerLayout L{};
  size_t o = kErrBytes;  // the region's error word first
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.recv_flag = take((size_t)P * 4);            // [P] u32: call number of source p's latest rows + counts
  L.ret_flag = take((size_t)P * 4);             // [P] u32: call number of owner q's latest returned rows
  L.done = take(2 * 4);                         // CTA-completion counters (dispatch, return)
  L.calls = take(4);                            // layer calls completed on this region (combine advances it)
  L.counts = take((size_t)P * El * 4);          // [P, El] rows source p sent for each local expert
  L.recv_off = take((size_t)P * 4);             // [P] source p's sorted position of its first row here
  L.recv_rows = take((size_t)P * cap * H * 2);  // [P, cap, H] 16-bit activation rows, per source
  L.ret_rows = take((size_t)cap * H * 2);       // [cap, H] fp16 down rows of this rank's picks, sorted order
  L.total = o;
  return L;
}

bool peer_desc_ok(const e4b_ep_peer_desc& p) {
  if (p.world < 1 || p.world > kMaxPeers || p.rank < 0 || p.rank >= p.world) return false;
  if (p.local_experts <= 0 || (int64_t)p.local_experts * p.world > 1024) return false;
  if (p.rows_per_rank <= 0 || p.hidden <= 0 || p.hidden % 64) return false;
  if ((int64_t)p.rows_per_rank * p.world > (1 << 30)) return false;
  if (!is_act_dtype(p.act_dtype) || !p.peers) return false;
  for (int q = 0; q < p.world; ++q)
    if (!p.peers[q] || (reinterpret_cast<uintptr_t>(p.peers[q]) & 255)) return false;
  return true;
}

struct PeerPtrs {
  char* base[kMaxPeers];
};

PeerPtrs peer_ptrs(const e4b_ep_peer_desc& p) {
  PeerPtrs r{};
  for (int q = 0; q < p.world; ++q) r.base[q] = static_cast<char*>(p.peers[q]);
  return r;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Called by every thread of every CTA after its peer stores: the last CTA to finish
// publishes the call number `epoch` in flag slot `slot` of every peer region (flags at `flag_off`).
__device__ void publish_when_last(unsigned* done, const PeerPtrs& peers, int P, size_t flag_off, int slot,
                                  unsigned epoch) {
  __shared__ int s_last;
  __threadfence_system();  // this thread's stores reach the peers before the count
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  if ((int)threadIdx.x < P)
    st_release_sys(reinterpret_cast<unsigned*>(peers.base[threadIdx.x] + flag_off) + slot, epoch);
  if (threadIdx.x == 0) *done = 0;  // ready for the next call (kernels on this stream are ordered)
}

// One 16-bit row of vec 16-byte units, copied by a warp with four loads in flight per lane
// before their stores (the stores may cross NVLink).
__device__ __forceinline__ void copy_row_warp(const uint4* __restrict__ src, uint4* __restrict__ dst, int vec,
                                              int lane) {
  int v = lane;
  for (; v + 96 < vec; v += 128) {
    const uint4 a = src[v], b = src[v + 32], c = src[v + 64], d = src[v + 96];
    dst[v] = a;
    dst[v + 32] = b;
    dst[v + 64] = c;
    dst[v + 96] = d;
  }
  for (; v < vec; v += 32) dst[v] = src[v];
}

struct PushArgs {
  PeerPtrs peers;
  PeerLayout L;
  int P, rank, El, cap, vec;  // vec = H / 8 (16-byte units per row)
  const unsigned* calls;      // this call publishes *calls + 1
  const uint4* hidden;
  const int32_t* sorted_token;
  const int32_t* offsets;     // [E+1] global expert segments of this rank's sorted picks
  int R;
  unsigned* done;
};

// Dispatch: sorted row r (global expert e, owner q = e / El) is stored at row
// r - offsets[q*El] of this rank's block in q's region; CTA 0 also stores the
// per-expert counts and the send offset; the last CTA raises the arrival flags.
__global__ void __launch_bounds__(256) ep_push_rows_kernel(PushArgs a) {
  __shared__ int s_bound[kMaxPeers + 1];
  const int tid = threadIdx.x;
  if (tid <= a.P) s_bound[tid] = a.offsets[tid * a.El];
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int i = tid; i < a.P * a.El; i += blockDim.x) {
      const int q = i / a.El, e = i - q * a.El;
      reinterpret_cast<int*>(a.peers.base[q] + a.L.counts)[a.rank * a.El + e] = a.offsets[i + 1] - a.offsets[i];
    }
    if (tid < a.P) reinterpret_cast<int*>(a.peers.base[tid] + a.L.recv_off)[a.rank] = s_bound[tid];
  }
  const int lane = tid & 31;
  for (int r = blockIdx.x * 8 + (tid >> 5); r < a.R; r += gridDim.x * 8) {
    int q = 0;
    while (q + 1 < a.P && r >= s_bound[q + 1]) ++q;
    const int j = r - s_bound[q];
    const uint4* src = a.hidden + (int64_t)a.sorted_token[r] * a.vec;
    uint4* dst = reinterpret_cast<uint4*>(a.peers.base[q] + a.L.recv_rows) + ((int64_t)a.rank * a.cap + j) * a.vec;
    copy_row_warp(src, dst, a.vec, lane);
  }
  publish_when_last(a.done, a.peers, a.P, a.L.recv_flag, a.rank, *a.calls + 1);
}

// One CTA: bounded wait until every source's flag reaches this call's number (*calls + 1),
// then copy the region's counts and offsets into local storage; sources that never arrived
// count 0. With `advance` (the last step of a call), thread 0 records the call as complete.
__global__ void __launch_bounds__(256) ep_peer_wait_kernel(const unsigned* flags, int P, unsigned* calls, int advance,
                                                           const int* src, int El, int* dst, const int* off_src,
                                                           int* off_dst, int* err) {
  __shared__ int s_dead[kMaxPeers];
  const int tid = threadIdx.x;
  const unsigned epoch = *calls + 1;
  if (tid < P) {
    int dead = 1;
    for (int i = 0; i < kPeerWaitPolls; ++i) {
      if ((int)(ld_acquire_sys(flags + tid) - epoch) >= 0) {
        dead = 0;
        break;
      }
      __nanosleep(256);
    }
    if (dead) raise_error(err, E4B_ERR_TIMEOUT);
    s_dead[tid] = dead;
  }
  __syncthreads();
  if (advance && tid == 0) *calls = epoch;
  if (!dst) return;
  for (int i = tid; i < P * El; i += blockDim.x) {
    const int p = i / El;
    dst[i] = s_dead[p] ? 0 : *reinterpret_cast<const volatile int*>(src + i);
  }
  if (tid < P) off_dst[tid] = s_dead[tid] ? 0 : *reinterpret_cast<const volatile int*>(off_src + tid);
}

// gather_convert bounded by the device row count: rows [0, *total) only.
__global__ void __launch_bounds__(256) ep_gather_convert_kernel(ConvertArgs c, const int32_t* __restrict__ rows_map,
                                                                const int32_t* __restrict__ total) {
  const int n = min(c.rows, *total);
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < n; r += gridDim.x * 8) {
    const int64_t src = rows_map[r];
    convert_rows_to_f16(reinterpret_cast<const char*>(c.src) + src * c.K * 2, c.src_dtype, c.dst + (int64_t)r * c.K,
                        c.scale + r, 1, c.K, 0, 1);
  }
}

struct ReturnArgs {
  PeerPtrs peers;
  PeerLayout L;
  int P, rank, cap, vec;
  const unsigned* calls;
  const uint4* down_rows;     // [R] expert-major fp16 rows
  const int32_t* map;         // expert-major row -> p * cap + j
  const int32_t* total;       // rows received
  const int32_t* recv_off;    // [P] local copy of the sources' send offsets
  unsigned* done;
};

// Return: expert-major row r came from source p as its row j; it goes to row
// recv_off[p] + j of p's return block. The last CTA raises the return flags.
__global__ void __launch_bounds__(256) ep_return_rows_kernel(ReturnArgs a) {
  const int lane = threadIdx.x & 31;
  const int n = *a.total;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < n; r += gridDim.x * 8) {
    const int sidx = a.map[r];
    const int p = sidx / a.cap, j = sidx - p * a.cap;
    const uint4* src = a.down_rows + (int64_t)r * a.vec;
    uint4* dst = reinterpret_cast<uint4*>(a.peers.base[p] + a.L.ret_rows) + (int64_t)(a.recv_off[p] + j) * a.vec;
    copy_row_warp(src, dst, a.vec, lane);
  }
  publish_when_last(a.done, a.peers, a.P, a.L.ret_flag, a.rank, *a.calls + 1);
}

// What the expert side needs to read from and write to peer regions.
struct PeerCtx {
  PeerPtrs peers;
  PeerLayout L;
  const e4b_ep_peer_desc* pd;
  int32_t* counts_local;  // [P, El]
  int32_t* off_local;     // [P]
};

size_t peer_extra_bytes(int P, int El) { return align_up((size_t)P * El * 4, 256) + align_up((size_t)P * 4, 256); }

// The expert side of one layer: plan, convert, the fused expert stages, and either the
// down rows in received order (t->out) or, with a peer context, stores into the sources'
// return blocks.
e4b_status ep_experts_run(const e4b_moe_desc& d, int world, const int32_t* recv_counts, const e4b_moe_tensors* t,
                          void* workspace, const EpLayout& L, int regime_rows, const PeerCtx* peer, cudaStream_t s) {
  const int R = d.tokens, El = d.num_experts, H = d.hidden, I = d.intermediate;
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws);
  if (cudaMemsetAsync(err, 0, sizeof(int), s) != cudaSuccess) return E4B_ERR_CUDA;
  mark_stage(t, 0, s);
  if (peer) {
    const char* own = peer->peers.base[peer->pd->rank];
    ep_peer_wait_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const unsigned*>(own + peer->L.recv_flag), world,
                                          reinterpret_cast<unsigned*>(const_cast<char*>(own) + peer->L.calls), 0,
                                          reinterpret_cast<const int*>(own + peer->L.counts), El,
                                          peer->counts_local, reinterpret_cast<const int*>(own + peer->L.recv_off),
                                          peer->off_local, reinterpret_cast<int*>(peer->peers.base[peer->pd->rank]));
    if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
    recv_counts = peer->counts_local;
  }
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
  if (peer) {
    pl.src_stride = peer->pd->rows_per_rank;
    pl.partial = 1;
  }
  ep_plan_kernel<<<1, 1024, 0, s>>>(pl);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  if (R == 0) {
    mark_stage(t, 6, s);
    return E4B_OK;
  }
  __half* x16 = reinterpret_cast<__half*>(ws + L.x16);
  float* x_scale = reinterpret_cast<float*>(ws + L.x_scale);
  ConvertArgs cv{};
  cv.src = peer ? static_cast<const void*>(peer->peers.base[peer->pd->rank] + peer->L.recv_rows) : t->hidden;
  cv.src_dtype = d.act_dtype;
  cv.dst = x16;
  cv.scale = x_scale;
  cv.rows = R;
  cv.K = H;
  e4b_status st = E4B_OK;
  if (peer) {
    ep_gather_convert_kernel<<<conv_ctas_for(R, 8), 256, 0, s>>>(
        cv, pl.map, pl.offsets + El);
    if ((st = launch_status()) != E4B_OK) return st;
  } else if ((st = launch_gather_convert(cv, pl.map, s)) != E4B_OK) {
    return st;
  }
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
  x.use_umma = umma_worthwhile(regime_rows, El) &&
               umma_eligible(regime_rows, 1, El, H, I, d.has_gate, d.act_dtype, d.lora_rank);
  x.h = ws + L.h;
  x.down_rows = ws + L.down_rows;
  x.xa_gu = reinterpret_cast<float*>(ws + L.xa_gu);
  x.xa_dn = reinterpret_cast<float*>(ws + L.xa_dn);
  x.umma_scratch = ws + L.umma;
  x.err = err;
  if ((st = run_expert_stages(d, t, x, s)) != E4B_OK) return st;
  if (peer) {
    ReturnArgs ra{};
    ra.peers = peer->peers;
    ra.L = peer->L;
    ra.P = world;
    ra.rank = peer->pd->rank;
    ra.cap = peer->pd->rows_per_rank;
    ra.vec = H / 8;
    ra.calls = reinterpret_cast<const unsigned*>(peer->peers.base[peer->pd->rank] + peer->L.calls);
    ra.down_rows = static_cast<const uint4*>(x.down_rows);
    ra.map = pl.map;
    ra.total = pl.offsets + El;
    ra.recv_off = peer->off_local;
    ra.done = reinterpret_cast<unsigned*>(peer->peers.base[peer->pd->rank] + peer->L.done) + 1;
    ep_return_rows_kernel<<<rows_ctas(R), 256, 0, s>>>(ra);
  } else {
    ep_scatter_rows_kernel<<<rows_ctas(R), 256, 0, s>>>(static_cast<const uint4*>(x.down_rows), pl.map, R, H / 8,
                                                        static_cast<uint4*>(t->out));
  }
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  mark_stage(t, 6, s);
  return E4B_OK;
}

e4b_status check_expert_side(const e4b_moe_desc& d, int world, const e4b_moe_tensors* t) {
  if (!ep_desc_ok(d, world)) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(d.act_dtype) || d.out_dtype != E4B_F16) return E4B_ERR_UNSUPPORTED;
  if (d.hidden % 64 || d.intermediate % 64) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank < 0 || d.lora_rank > kLoraMaxRank) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank > 0 && !is_any_dtype(d.lora_dtype)) return E4B_ERR_UNSUPPORTED;
  if (e4b_status fs = check_weight_format(d)) return fs;
  if (!t->gate_up_packed || !t->gate_up_absmax || !t->down_packed || !t->down_absmax) return E4B_ERR_INVALID_ARG;
  if (d.lora_rank > 0 && (!t->gate_up_lora_A || !t->gate_up_lora_B || !t->down_lora_A || !t->down_lora_B))
    return E4B_ERR_INVALID_ARG;
  if (!aligned16(t->gate_up_packed) || !aligned16(t->down_packed)) return E4B_ERR_ALIGNMENT;
  return E4B_OK;
}

// The expert-side descriptor with the received-row capacity as its row count.
e4b_moe_desc peer_capacity_desc(const e4b_ep_peer_desc& pd, const e4b_moe_desc& local) {
  e4b_moe_desc d = local;
  d.tokens = pd.world * pd.rows_per_rank;
  return d;
}

}  // namespace

}  // namespace e4b

extern "C" size_t e4b_ep_experts_workspace_bytes(const e4b_moe_desc* local, int world) {
  if (!local || !ep_desc_ok(*local, world)) return 0;
  return ep_layout(*local, world).total;
}

extern "C" e4b_status e4b_ep_experts(const e4b_moe_desc* local, int world, const int32_t* recv_counts,
                                     const e4b_moe_tensors* t, void* workspace, size_t workspace_bytes, void* stream) {
  if (!local || !t || !ep_desc_ok(*local, world)) return E4B_ERR_INVALID_ARG;
  const e4b_moe_desc& d = *local;
  if (e4b_status cs = check_expert_side(d, world, t)) return cs;
  const int R = d.tokens;
  if (!recv_counts) return E4B_ERR_INVALID_ARG;
  if (R > 0 && (!t->hidden || !t->out)) return E4B_ERR_INVALID_ARG;
  if (R > 0 && (!aligned16(t->hidden) || !aligned16(t->out))) return E4B_ERR_ALIGNMENT;
  const EpLayout L = ep_layout(d, world);
  if (!workspace || workspace_bytes < L.total) return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace)) return E4B_ERR_ALIGNMENT;
  return ep_experts_run(d, world, recv_counts, t, workspace, L, R, nullptr, (cudaStream_t)stream);
}

// ---- peer-memory entry points ----

extern "C" size_t e4b_ep_comm_bytes(int world, int local_experts, int rows_per_rank, int hidden) {
  if (world < 1 || world > E4B_EP_MAX_PEERS || local_experts <= 0 || rows_per_rank <= 0 || hidden <= 0) return 0;
  if ((int64_t)local_experts * world > 1024 || (int64_t)rows_per_rank * world > (1 << 30)) return 0;
  return peer_layout(world, local_experts, rows_per_rank, hidden).total;
}

namespace {
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  }
  return fn;
}
}  // namespace

extern "C" e4b_status e4b_ipc_export(const void* ptr, void* handle_host, size_t* offset_host) {
  static_assert(sizeof(cudaIpcMemHandle_t) <= E4B_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle_host || !offset_host) return E4B_ERR_INVALID_ARG;
  GetAddressRangeFn range = address_range_fn();
  if (!range) return E4B_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return E4B_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return E4B_ERR_CUDA;
  memset(handle_host, 0, E4B_IPC_HANDLE_BYTES);
  memcpy(handle_host, &h, sizeof(h));
  *offset_host = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return E4B_OK;
}

extern "C" e4b_status e4b_ipc_open(const void* handle_host, size_t offset, void** ptr_host) {
  if (!handle_host || !ptr_host) return E4B_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle_host, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return E4B_ERR_CUDA;
  *ptr_host = static_cast<char*>(base) + offset;
  return E4B_OK;
}

extern "C" e4b_status e4b_ipc_close(void* ptr, size_t offset) {
  if (!ptr) return E4B_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) == cudaSuccess ? E4B_OK : E4B_ERR_CUDA;
}

extern "C" size_t e4b_ep_dispatch_peer_workspace_bytes(int T, int k, int E) {
  return e4b_ep_dispatch_workspace_bytes(T, k, E);
}

extern "C" e4b_status e4b_ep_dispatch_peer(const e4b_ep_peer_desc* pd, const void* hidden, const int64_t* topk_idx,
                                           int T, int k, int32_t* inv, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  if (!pd || !peer_desc_ok(*pd)) return E4B_ERR_INVALID_ARG;
  const int P = pd->world, El = pd->local_experts, E = P * El, H = pd->hidden;
  if (T < 0 || k <= 0 || k > 32 || k > E || (int64_t)T * k > pd->rows_per_rank) return E4B_ERR_INVALID_ARG;
  if (T > 0 && (!hidden || !topk_idx || !inv)) return E4B_ERR_INVALID_ARG;
  if (T > 0 && !aligned16(hidden)) return E4B_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < e4b_ep_dispatch_workspace_bytes(T, k, E)) return E4B_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + kErrBytes);
  int32_t* sorted_token = reinterpret_cast<int32_t*>(ws + kErrBytes + align_up((size_t)(E + 1) * 4, 256));
  char* own = static_cast<char*>(pd->peers[pd->rank]);
  const PeerLayout L = peer_layout(P, El, pd->rows_per_rank, H);
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
  pa.err = reinterpret_cast<int*>(own);  // the region's error word
  pa.reset_err = 0;  // the error word is sticky: only e4b_read_device_error clears it
  e4b_status st = launch_permute(pa, s);
  if (st != E4B_OK) return st;
  PushArgs a{};
  a.peers = peer_ptrs(*pd);
  a.L = L;
  a.P = P;
  a.rank = pd->rank;
  a.El = El;
  a.cap = pd->rows_per_rank;
  a.vec = H / 8;
  a.calls = reinterpret_cast<const unsigned*>(own + L.calls);
  a.hidden = static_cast<const uint4*>(hidden);
  a.sorted_token = sorted_token;
  a.offsets = offsets;
  a.R = T * k;
  a.done = reinterpret_cast<unsigned*>(own + L.done);
  ep_push_rows_kernel<<<rows_ctas(T * k), 256, 0, s>>>(a);
  return launch_status();
}

extern "C" size_t e4b_ep_experts_peer_workspace_bytes(const e4b_ep_peer_desc* pd, const e4b_moe_desc* local) {
  if (!pd || !local || !peer_desc_ok(*pd) || local->num_experts != pd->local_experts) return 0;
  const e4b_moe_desc d = peer_capacity_desc(*pd, *local);
  if (!ep_desc_ok(d, pd->world)) return 0;
  return ep_layout(d, pd->world).total + peer_extra_bytes(pd->world, pd->local_experts);
}

extern "C" e4b_status e4b_ep_experts_peer(const e4b_ep_peer_desc* pd, const e4b_moe_desc* local,
                                          const e4b_moe_tensors* t, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (!pd || !local || !t || !peer_desc_ok(*pd)) return E4B_ERR_INVALID_ARG;
  if (local->num_experts != pd->local_experts || local->hidden != pd->hidden || local->act_dtype != pd->act_dtype)
    return E4B_ERR_INVALID_ARG;
  const e4b_moe_desc d = peer_capacity_desc(*pd, *local);
  if (e4b_status cs = check_expert_side(d, pd->world, t)) return cs;
  const EpLayout L = ep_layout(d, pd->world);
  if (!workspace || workspace_bytes < L.total + peer_extra_bytes(pd->world, pd->local_experts))
    return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace)) return E4B_ERR_ALIGNMENT;
  PeerCtx ctx{};
  ctx.peers = peer_ptrs(*pd);
  ctx.L = peer_layout(pd->world, pd->local_experts, pd->rows_per_rank, pd->hidden);
  ctx.pd = pd;
  char* extra = static_cast<char*>(workspace) + L.total;
  ctx.counts_local = reinterpret_cast<int32_t*>(extra);
  ctx.off_local = reinterpret_cast<int32_t*>(extra + align_up((size_t)pd->world * pd->local_experts * 4, 256));
  const int hint = local->tokens < 0 ? 0 : (local->tokens > d.tokens ? d.tokens : local->tokens);
  return ep_experts_run(d, pd->world, nullptr, t, workspace, L, hint, &ctx, (cudaStream_t)stream);
}

extern "C" e4b_status e4b_ep_combine_peer(const e4b_ep_peer_desc* pd, const int32_t* inv, const void* topk_w,
                                          int w_dtype, int T, int k, void* out, int out_dtype, void* stream) {
  if (!pd || !peer_desc_ok(*pd)) return E4B_ERR_INVALID_ARG;
  if (T < 0 || k <= 0 || (int64_t)T * k > pd->rows_per_rank) return E4B_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  char* own = static_cast<char*>(pd->peers[pd->rank]);
  const PeerLayout L = peer_layout(pd->world, pd->local_experts, pd->rows_per_rank, pd->hidden);
  ep_peer_wait_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const unsigned*>(own + L.ret_flag), pd->world,
                                        reinterpret_cast<unsigned*>(own + L.calls), 1, nullptr, pd->local_experts, nullptr, nullptr, nullptr,
                                        reinterpret_cast<int*>(own));
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  return e4b_combine(own + L.ret_rows, E4B_F16, inv, topk_w, w_dtype, T, k, pd->hidden, out, out_dtype, stream);
}
