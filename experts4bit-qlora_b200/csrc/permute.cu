// Permutation (R2): the device-side replacement for engines/fast.py:126-135.
//
// order = argsort(flat top-k ids, stable); counts = bincount; offsets =
// exclusive scan -- computed in one CTA of 32 warps with no host round trip (large
// inputs: the same passes over the grid, below).
// Each warp owns a contiguous segment of the flat array, so ranks within an
// expert follow flat order exactly (stable): pass 1 counts per (warp, expert),
// pass 2 scans expert-major / warp-minor, pass 3 re-walks each segment in order
// and places every entry with __match_any_sync ranks.
#include "common.cuh"
#include "permute.cuh"

namespace e4b {

__device__ __forceinline__ int block_exclusive_scan(int v, int* smem_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? smem_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) smem_warp[lane] = w;
  }
  __syncthreads();
  const int before = (warp ? smem_warp[warp - 1] : 0) + x - v;
  if (total) *total = smem_warp[nw - 1];
  __syncthreads();
  return before;
}

// Whole permutation in one warp when T*k <= 32 (decode): lane i holds flat entry i;
// ranks, counts, offsets and the active list come from shuffles, with no block
// barriers and no shared memory.
__device__ void permute_one_warp(const PermuteArgs& a) {
  const int lane = threadIdx.x & 31;
  const int E = a.E, n = a.T * a.k;
  if (a.reset_err && lane == 0 && a.err) *a.err = 0;
  __syncwarp();
  int e = 0x7fffffff;
  if (lane < n) {
    e = stack_expert(a.topk_idx[lane], a.emap, a.routed, E, a.err, true);
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const bool valid = lane < n;
  const bool lead = valid && (peers & ((1u << lane) - 1u)) == 0;  // first entry of its expert
  const int cnt = __popc(peers);
  int below = 0, distinct_below = 0;  // entries / experts with a smaller id
  for (int j = 0; j < n; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e, j);
    below += ej < e;
  }
  const unsigned leaders = __ballot_sync(0xffffffffu, lead);
  for (int j = 0; j < n; ++j) {
    const int ej = __shfl_sync(0xffffffffu, e, j);
    distinct_below += ((leaders >> j) & 1u) && ej < e;
  }
  if (valid) {
    const int pos = below + __popc(peers & ((1u << lane) - 1u));
    if (a.order) a.order[pos] = lane;
    if (a.inv) a.inv[lane] = pos;
    if (a.sorted_token) a.sorted_token[pos] = lane / a.k;
    if (lead && a.active) a.active[distinct_below] = e;
  }
  if (lane == 0 && a.num_active) *a.num_active = __popc(leaders);
  // per-expert prefix arrays over all E experts
  for (int x0 = 0; x0 <= E; x0 += 32) {  // warp-uniform trip count: every shuffle has all lanes
    const int x = x0 + lane;
    int off = 0, ta = 0, tb = 0;
    for (int j = 0; j < 32; ++j) {
      const int ej = __shfl_sync(0xffffffffu, e, j);
      const int cj = __shfl_sync(0xffffffffu, cnt, j);
      off += (j < n) && ej < x;
      if (((leaders >> j) & 1u) && ej < x) {
        ta += (cj + a.tile_a - 1) / max(a.tile_a, 1);
        tb += (cj + a.tile_b - 1) / max(a.tile_b, 1);
      }
    }
    if (x <= E) {
      a.offsets[x] = off;
      if (a.tile_start_a) a.tile_start_a[x] = ta;
      if (a.tile_start_b) a.tile_start_b[x] = tb;
    }
  }
}

__global__ void __launch_bounds__(1024)
permute_kernel(PermuteArgs a) {
  if (blockIdx.x > 0) {  // conversion CTAs: one row per warp
    convert_rows_to_f16(a.conv.src, a.conv.src_dtype, a.conv.dst, a.conv.scale, a.conv.rows, a.conv.K,
                        (blockIdx.x - 1) * (blockDim.x >> 5) + (threadIdx.x >> 5), a.conv_ctas * (blockDim.x >> 5));
    return;
  }
  if (a.T * a.k <= 32) {
    if (threadIdx.x < 32) permute_one_warp(a);
    return;
  }
  extern __shared__ int wc[];           // [32][E]
  __shared__ int s_scan[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int E = a.E;
  const int n = a.T * a.k;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wc[i] = 0;
  if (a.reset_err && threadIdx.x == 0 && a.err) *a.err = 0;
  __syncthreads();
  const int seg = (n + 31) / 32;
  const int s0 = min(n, warp * seg), s1 = min(n, s0 + seg);
  const unsigned lt = (1u << lane) - 1u;
  // The segment's first kCache x 32 entries are loaded once, all in flight, and kept in registers
  // (fully unrolled steps, so the indices are static) for pass 3; longer segments reload the rest.
  constexpr int kCache = 24;
  int ec[kCache];
  auto load_entry = [&](int i, bool flag) -> int {
    return stack_expert(a.topk_idx[i], a.emap, a.routed, E, a.err, flag);
  };
#pragma unroll
  for (int it = 0; it < kCache; ++it) {
    const int i = s0 + it * 32 + lane;
    ec[it] = i < s1 ? load_entry(i, true) : 0;
  }
  auto count_step = [&](int base, int e) {  // pass 1 on the 32 entries at base
    const bool valid = base + lane < s1;
    const unsigned act = __ballot_sync(0xffffffffu, valid);
    const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1) & act;
    if (valid && (peers & lt) == 0) wc[warp * E + e] += __popc(peers);
    __syncwarp();
  };
  // pass 1: per-warp counts
#pragma unroll
  for (int it = 0; it < kCache; ++it)
    if (s0 + it * 32 < s1) count_step(s0 + it * 32, ec[it]);
  for (int base = s0 + kCache * 32; base < s1; base += 32)
    count_step(base, base + lane < s1 ? load_entry(base + lane, true) : 0);
  __syncthreads();
  // pass 2: counts, offsets, per-warp bases (one expert per thread, E <= 1024)
  {
    const int e = threadIdx.x;
    int c = 0;
    if (e < E) {
      for (int w = 0; w < 32; ++w) {
        const int t = wc[w * E + e];
        wc[w * E + e] = c;           // exclusive prefix over warps
        c += t;
      }
    }
    int tot;
    const int off = block_exclusive_scan(c, s_scan, &tot);
    if (e < E) {
      a.offsets[e] = off;
      for (int w = 0; w < 32; ++w) wc[w * E + e] += off;
    }
    if (threadIdx.x == 0) a.offsets[E] = n;
    // active-expert list and tile prefixes
    const int pos = block_exclusive_scan(c > 0 ? 1 : 0, s_scan, &tot);
    if (e < E && c > 0 && a.active) a.active[pos] = e;
    if (threadIdx.x == 0 && a.num_active) *a.num_active = tot;
    for (int j = 0; j < 2; ++j) {
      int* ts = j == 0 ? a.tile_start_a : a.tile_start_b;
      const int bm = j == 0 ? a.tile_a : a.tile_b;
      if (!ts) continue;
      const int nt = e < E ? (c + bm - 1) / bm : 0;
      const int p = block_exclusive_scan(nt, s_scan, &tot);
      if (e < E) ts[e] = p;
      if (threadIdx.x == 0) ts[E] = tot;
    }
  }
  __syncthreads();
  // pass 3: place every entry (stable)
  auto place_step = [&](int base, int e) {
    const int i = base + lane;
    const bool valid = i < s1;
    const unsigned act = __ballot_sync(0xffffffffu, valid);
    const unsigned peers = __match_any_sync(0xffffffffu, valid ? e : -1) & act;
    int pos = 0;
    if (valid) pos = wc[warp * E + e] + __popc(peers & lt);
    __syncwarp();
    if (valid && (peers & lt) == 0) wc[warp * E + e] += __popc(peers);
    __syncwarp();
    if (valid) {
      if (a.order) a.order[pos] = i;
      if (a.inv) a.inv[i] = pos;
      if (a.sorted_token) a.sorted_token[pos] = i / a.k;
    }
  };
#pragma unroll
  for (int it = 0; it < kCache; ++it)
    if (s0 + it * 32 < s1) place_step(s0 + it * 32, ec[it]);
  for (int base = s0 + kCache * 32; base < s1; base += 32)
    place_step(base, base + lane < s1 ? load_entry(base + lane, false) : 0);
}

size_t permute_smem_bytes(int E) { return (size_t)32 * E * sizeof(int); }

// ---- multi-CTA permutation for large inputs --------------------------------------------------
// The one-CTA kernel walks every entry on one SM. Above kMultiMin entries the same three passes
// run over the grid: segments of kSeg consecutive flat entries (one warp each) count per expert
// into global scratch; one CTA scans expert-major / segment-minor into the offsets, the tile
// prefixes, the active list and each segment's base per expert; every warp then re-walks its
// segment and places its entries with __match_any_sync ranks. Segments are contiguous and
// ordered, so ranks within an expert follow flat order: the same stable result as the one-CTA
// kernel.
constexpr int kMultiMin = 8192;
constexpr int kSeg = 256;

size_t permute_scratch_bytes(int64_t n, int E) {
  if (n <= kMultiMin) return 0;
  return (size_t)((n + kSeg - 1) / kSeg) * E * sizeof(int32_t);
}

__global__ void __launch_bounds__(1024) permute_count_kernel(PermuteArgs a, int nseg, int count_ctas) {
  if ((int)blockIdx.x >= count_ctas) {  // conversion CTAs: one row per warp
    convert_rows_to_f16(a.conv.src, a.conv.src_dtype, a.conv.dst, a.conv.scale, a.conv.rows, a.conv.K,
                        (blockIdx.x - count_ctas) * (blockDim.x >> 5) + (threadIdx.x >> 5),
                        a.conv_ctas * (blockDim.x >> 5));
    return;
  }
  extern __shared__ int wc[];  // [32][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, E = a.E, n = a.T * a.k;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int seg = blockIdx.x * 32 + warp;
  if (seg < nseg) {
    const int s0 = seg * kSeg, s1 = min(n, s0 + kSeg);
    const unsigned lt = (1u << lane) - 1u;
    int64_t ids[kSeg / 32];  // the segment's expert ids, all loads in flight at once
#pragma unroll
    for (int j = 0; j < kSeg / 32; ++j) ids[j] = s0 + 32 * j + lane < s1 ? a.topk_idx[s0 + 32 * j + lane] : 0;
#pragma unroll
    for (int j = 0; j < kSeg / 32; ++j) {
      const int base = s0 + 32 * j;
      const int i = base + lane;
      const bool valid = i < s1;
      const int e = valid ? stack_expert(ids[j], a.emap, a.routed, E, a.err, true) : -1;
      const unsigned act = __ballot_sync(0xffffffffu, valid);
      const unsigned peers = __match_any_sync(0xffffffffu, e) & act;
      if (valid && (peers & lt) == 0) wc[warp * E + e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) {
    const int w = i / E, e = i - w * E;
    const int sg = blockIdx.x * 32 + w;
    if (sg < nseg) a.seg_scratch[(int64_t)sg * E + e] = wc[i];
  }
}

__global__ void __launch_bounds__(1024) permute_scan_kernel(PermuteArgs a, int nseg) {
  __shared__ int s_scan[32];
  const int E = a.E, n = a.T * a.k, e = threadIdx.x;
  // Prefix over segments, written back in place. Sixteen segments' counts are loaded before any
  // of their stores, so one memory round trip covers sixteen segments instead of one.
  constexpr int kB = 16;
  int c = 0;
  if (e < E) {
    for (int sg0 = 0; sg0 < nseg; sg0 += kB) {
      int v[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j) v[j] = sg0 + j < nseg ? a.seg_scratch[(int64_t)(sg0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < kB; ++j)
        if (sg0 + j < nseg) {
          a.seg_scratch[(int64_t)(sg0 + j) * E + e] = c;
          c += v[j];
        }
    }
  }
  int tot;
  const int off = block_exclusive_scan(c, s_scan, &tot);
  if (e < E) {
    a.offsets[e] = off;
    for (int sg0 = 0; sg0 < nseg; sg0 += kB) {
      int v[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j) v[j] = sg0 + j < nseg ? a.seg_scratch[(int64_t)(sg0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < kB; ++j)
        if (sg0 + j < nseg) a.seg_scratch[(int64_t)(sg0 + j) * E + e] = v[j] + off;
    }
  }
  if (threadIdx.x == 0) a.offsets[E] = n;
  const int pos = block_exclusive_scan(c > 0 ? 1 : 0, s_scan, &tot);
  if (e < E && c > 0 && a.active) a.active[pos] = e;
  if (threadIdx.x == 0 && a.num_active) *a.num_active = tot;
  for (int j = 0; j < 2; ++j) {
    int* ts = j == 0 ? a.tile_start_a : a.tile_start_b;
    const int bm = j == 0 ? a.tile_a : a.tile_b;
    if (!ts) continue;
    const int nt = e < E ? (c + bm - 1) / bm : 0;
    const int p = block_exclusive_scan(nt, s_scan, &tot);
    if (e < E) ts[e] = p;
    if (threadIdx.x == 0) ts[E] = tot;
  }
}

__global__ void __launch_bounds__(1024) permute_place_kernel(PermuteArgs a, int nseg) {
  extern __shared__ int wc[];  // [32][E]: this CTA's segments' running bases
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, E = a.E, n = a.T * a.k;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) {
    const int w = i / E, e = i - w * E;
    const int sg = blockIdx.x * 32 + w;
    wc[i] = sg < nseg ? a.seg_scratch[(int64_t)sg * E + e] : 0;
  }
  __syncthreads();
  const int seg = blockIdx.x * 32 + warp;
  if (seg >= nseg) return;
  const int s0 = seg * kSeg, s1 = min(n, s0 + kSeg);
  const unsigned lt = (1u << lane) - 1u;
  int64_t ids[kSeg / 32];
#pragma unroll
  for (int j = 0; j < kSeg / 32; ++j) ids[j] = s0 + 32 * j + lane < s1 ? a.topk_idx[s0 + 32 * j + lane] : 0;
#pragma unroll
  for (int j = 0; j < kSeg / 32; ++j) {
    const int base = s0 + 32 * j;
    const int i = base + lane;
    const bool valid = i < s1;
    const int e = valid ? stack_expert(ids[j], a.emap, a.routed, E, a.err, false) : -1;
    const unsigned act = __ballot_sync(0xffffffffu, valid);
    const unsigned peers = __match_any_sync(0xffffffffu, e) & act;
    int pos = 0;
    if (valid) pos = wc[warp * E + e] + __popc(peers & lt);
    __syncwarp();
    if (valid && (peers & lt) == 0) wc[warp * E + e] += __popc(peers);
    __syncwarp();
    if (valid) {
      if (a.order) a.order[pos] = i;
      if (a.inv) a.inv[i] = pos;
      if (a.sorted_token) a.sorted_token[pos] = i / a.k;
    }
  }
}

e4b_status launch_permute(const PermuteArgs& a, cudaStream_t s) {
  const int64_t n = (int64_t)a.T * a.k;
  if (a.seg_scratch && n > kMultiMin) {
    const int nseg = (int)((n + kSeg - 1) / kSeg);
    const int ctas = (nseg + 31) / 32;
    const size_t smem = permute_smem_bytes(a.E);
    if (smem > 48 * 1024) {
      if (cudaFuncSetAttribute(permute_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
              cudaSuccess ||
          cudaFuncSetAttribute(permute_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
              cudaSuccess)
        return E4B_ERR_CUDA;
    }
    permute_count_kernel<<<ctas + (a.conv.src ? a.conv_ctas : 0), 1024, smem, s>>>(a, nseg, ctas);
    permute_scan_kernel<<<1, 1024, 0, s>>>(a, nseg);
    permute_place_kernel<<<ctas, 1024, smem, s>>>(a, nseg);
    return launch_status();
  }
  const size_t smem = permute_smem_bytes(a.E);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return E4B_ERR_CUDA;
  }
  permute_kernel<<<1 + (a.conv.src ? a.conv_ctas : 0), 1024, smem, s>>>(a);
  return launch_status();
}

}  // namespace e4b

using namespace e4b;

extern "C" size_t e4b_permute_workspace_bytes(int T, int k, int E) {
  if (E < 0 || T < 0 || k < 0) return 0;
  return kErrBytes + permute_scratch_bytes((int64_t)T * k, E);
}

extern "C" e4b_status e4b_permute(const int64_t* topk_idx, int T, int k, int E, int32_t* order, int32_t* inv,
                                  int32_t* offsets, void* workspace, size_t workspace_bytes, void* stream) {
  if (T < 0 || k <= 0 || E <= 0 || E > 1024 || (int64_t)T * k > (1 << 30)) return E4B_ERR_INVALID_ARG;
  if (!offsets || (T > 0 && !topk_idx)) return E4B_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < e4b_permute_workspace_bytes(T, k, E)) return E4B_ERR_WORKSPACE;
  PermuteArgs a{};
  a.topk_idx = topk_idx;
  a.T = T;
  a.k = k;
  a.E = E;
  a.order = order;
  a.inv = inv;
  a.offsets = offsets;
  a.err = static_cast<int*>(workspace);
  a.reset_err = 0;  // the error word is sticky: only e4b_read_device_error clears it
  if (permute_scratch_bytes((int64_t)T * k, E))
    a.seg_scratch = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + kErrBytes);
  return launch_permute(a, (cudaStream_t)stream);
}
