// Whole expert layer in one launch for the bs=1..8 decode regime (NF4, no
// adapters): router (optional) -> permute -> gate_up GEMV + SwiGLU -> down GEMV
// -> weighted combine, the per-layer chain of experts4bit_qlora/engines/fast.py:100-160.
//
// Layout of the work (one CTA per SM, 16 warps):
//  * Router: the CTAs of a thread-block cluster split the (expert, token tile)
//    logit tasks, gather the peers' logits through distributed shared memory
//    and run the same ranked top-k; no grid-wide barrier.
//  * Items: every CTA streams a fixed list of items through a ring of shared
//    memory slots filled by per-row bulk copies (cp.async.bulk, mbarrier
//    completion). An item is 16 weight rows x up to 2048 K elements:
//      gate_up tile (8 gate + the 8 matching up rows of one expert), assigned
//        round-robin over the grid in expert-major order, so expert j's h is
//        complete at ~ (j + 1) / active of the gate_up phase;
//      down tile (the CTA's own output rows of one expert), placed in the
//        CTA's list two experts after that expert's gate_up tiles.
//    All 16 warps work on one item at a time, each on its own K blocks
//    (k-split), with the token / h fragments of its blocks in registers;
//    NF4 codes decode through a per-lane pair table (conflict-free LDS) into
//    mma.sync m16n8k16 (fp32 accumulation), the block absmax folded in fp32
//    per 64-element block. The 16 partial tiles are summed in warp order.
//  * gate_up epilogue: SwiGLU, h rows (fp16) to global memory, then a release
//    increment of the expert's tile counter.
//  * down: a CTA needs an expert's h only when it reaches that expert's down
//    tile; its control thread polls the counter (acquire, bounded) ahead of
//    time and bulk-copies the expert's h rows into shared memory.
//  * combine: each CTA owns whole output rows, so the fixed slot-order
//    weighted sum needs no further synchronisation.
// Counters live at a fixed offset of the workspace (kFlowSyncOffset), must be
// zero before the first launch and are zeroed again by the last CTA to finish.
// Every wait is bounded; a timeout raises E4B_ERR_TIMEOUT and the kernel runs to
// its end. Device errors go straight into the sticky workspace error word.
#include <cooperative_groups.h>

#include <mutex>

#include "convert.cuh"
#include "decode_layer.cuh"
#include "router.cuh"
#include "stream_core.cuh"

namespace e4b {

namespace {

using stream::lut2;
using stream::mma16816;
using stream::mma16816_zero;

constexpr int kFWarps = 16;
constexpr int kFThreads = kFWarps * 32;
constexpr int kFChunk = 2048;               // K elements per item
constexpr int kFPitch = 1024 + 32;          // bytes per weight row in a slot (bank shift of 8 per row)
constexpr int kFAPitch = 128 + 16;          // bytes per absmax row in a slot (bank shift of 4 per row)
constexpr int kFSlotW = 16 * kFPitch;
constexpr int kFSlot = kFSlotW + 16 * kFAPitch;  // 19200 B
constexpr int kFMaxT = 8;
constexpr int kFMaxR = kFlowMaxPicks;
constexpr int kFMaxItems = 1024;
constexpr int kFMaxLogits = 2048;
constexpr int kFMaxSlots = 12;
constexpr int kFLag = 2;                    // experts between an expert's gate_up tiles and its down tile
constexpr int kFLut = 256 * 128;
constexpr int kFTabInts = 1152;             // the kernel's int tables (1120 used)
constexpr int kSmemCap = 232448;

struct FlowArgs {
  const void* hidden;
  int act_dtype;
  const int64_t* topk_idx;
  const void* topk_w;
  int w_dtype;
  const int32_t* emap;  // optional routed id -> stack index
  int routed;
  const uint8_t* gu_packed;
  const float* gu_absmax;
  const uint8_t* dn_packed;
  const float* dn_absmax;
  int T, k, E, H, I, has_gate;
  void* out;
  int out_dtype;
  __half* h;            // [R, I] fp16 scratch
  unsigned* sync;       // [kFMaxR + 1]: tile counters per active expert, then the finished-CTA count
  int* err;             // sticky device error word
  const void* router_w;  // fused router when non-null
  int router_w_dtype, route_kind, renorm;
  int64_t* topk_idx_out;
  float* topk_w_out;
  // shared-memory plan (bytes), computed on the host
  int nslots, o_ring, o_x, o_h, o_logits, o_tab, o_items, o_red, o_dval, o_bars;
  int hpitch;           // halves per staged h row
  int drows;            // rows per pick in dval (the CTA's output rows, rounded up to 16)
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

template <typename T> __device__ __forceinline__ T out_cast(float v, int*) { return from_f32<T>(v); }
template <> __device__ __forceinline__ __half out_cast<__half>(float v, int* err) { return store_cast<__half>(v, err); }

// Item word: bit 31 down (else gate_up), bits 24-30 active expert, bits 8-23 tile, bits 0-7 chunk.
__device__ __forceinline__ unsigned item_word(bool down, int j, int tile, int ch) {
  return (down ? 0x80000000u : 0u) | ((unsigned)j << 24) | ((unsigned)tile << 8) | (unsigned)ch;
}

struct Item {
  bool down;
  int j, tile, ch;
};
__device__ __forceinline__ Item item_of(unsigned w) {
  return Item{(w >> 31) != 0, (int)((w >> 24) & 127), (int)((w >> 8) & 0xFFFF), (int)(w & 0xFF)};
}

// Output rows [r0, r1) of CTA c: an even split of H over the grid.
__device__ __forceinline__ void my_rows(int H, int& r0, int& r1) {
  r0 = (int)(((int64_t)blockIdx.x * H) / gridDim.x);
  r1 = (int)(((int64_t)(blockIdx.x + 1) * H) / gridDim.x);
}

// Copies of one item into its slot (all 32 lanes of the calling warp): lane m < 16 copies weight
// row m's chunk, lane 16 + m its absmax; rows past the tile's valid count are left as they are.
__device__ __forceinline__ void issue_item(const FlowArgs& a, unsigned w, char* slot, uint64_t* bar,
                                           const int* act_e, int r0, int nr) {
  const int lane = threadIdx.x & 31;
  const Item it = item_of(w);
  const int e = act_e[it.j];
  const int K = it.down ? a.I : a.H;
  const int kc = min(kFChunk, K - it.ch * kFChunk);
  const uint32_t cb = kc / 2, ab = kc / 16;
  int nvalid;
  if (it.down) nvalid = min(16, nr - 16 * it.tile);
  else nvalid = 16;
  if (lane == 0) mbar_arrive_expect_tx(bar, nvalid * (cb + ab));
  __syncwarp();
  const int m = lane & 15;
  if (m < nvalid) {
    int64_t row;
    if (it.down) {
      row = (int64_t)e * a.H + r0 + 16 * it.tile + m;
    } else {
      const int n1 = a.has_gate ? 2 * a.I : a.I;
      row = a.has_gate ? (int64_t)e * n1 + (m < 8 ? 8 * it.tile + m : a.I + 8 * it.tile + m - 8)
                       : (int64_t)e * n1 + 16 * it.tile + m;
    }
    if (lane < 16) {
      const uint8_t* src = (it.down ? a.dn_packed : a.gu_packed) + row * (K / 2) + (int64_t)it.ch * (kFChunk / 2);
      bulk_g2s(slot + m * kFPitch, src, cb, bar);
    } else {
      const char* src = reinterpret_cast<const char*>(it.down ? a.dn_absmax : a.gu_absmax) + row * (K / 16) +
                        (int64_t)it.ch * (kFChunk / 16);
      bulk_g2s(slot + kFSlotW + m * kFAPitch, src, ab, bar);
    }
  }
}

// Control thread: bulk-copy expert j's h rows into shared memory once all its gate_up tiles are
// published. `seen` is a counter value the caller already read (relaxed); when it is short of
// complete and `blocking`, this waits (acquire, bounded). Returns whether the copy was requested.
__device__ bool request_h(const FlowArgs& a, int j, bool blocking, unsigned seen, int* hreq, uint64_t* hbar,
                          const int* act_row0, const int* act_cnt, __half* hs) {
  if (hreq[j]) return true;
  const unsigned need = (unsigned)((a.has_gate ? 2 * a.I : a.I) / 16);
  bool ok = seen >= need;
  if (ok) {
    fence_acq_rel_gpu();  // the relaxed observation becomes an acquire
  } else {
    if (!blocking) return false;
    for (uint32_t i = 0; i < kMaxSpins; ++i) {
      if (ld_acquire_gpu(&a.sync[j]) >= need) {
        ok = true;
        break;
      }
      __nanosleep(32);
    }
  }
  hreq[j] = 1;
  if (!ok) {  // gave up: flag it, complete the barrier without data
    raise_error(a.err, E4B_ERR_TIMEOUT);
    mbar_arrive(&hbar[j]);
    return true;
  }
  fence_proxy_async_global();  // the acquired h stores, ordered before the async-proxy reads
  const int n = act_cnt[j], r0 = act_row0[j];
  mbar_arrive_expect_tx(&hbar[j], (uint32_t)(n * a.I * 2));
  for (int c = 0; c < n; ++c)
    bulk_g2s(hs + (int64_t)(r0 + c) * a.hpitch, a.h + (int64_t)(r0 + c) * a.I, (uint32_t)(a.I * 2), &hbar[j]);
  return true;
}

template <typename OutT>
__global__ void __launch_bounds__(kFThreads, 1) nf4_decode_flow_kernel(const FlowArgs a) {
  extern __shared__ __align__(1024) char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, q = lane & 3;
  const int G = gridDim.x;
  const int T = a.T, k = a.k, R = T * k;
  const int n1 = a.has_gate ? 2 * a.I : a.I;
  const uint32_t lane4 = (uint32_t)lane << 2;

  char* lut = smem;
  char* ring = smem + a.o_ring;
  __half* xs = reinterpret_cast<__half*>(smem + a.o_x);
  __half* hs = reinterpret_cast<__half*>(smem + a.o_h);
  int* tb = reinterpret_cast<int*>(smem + a.o_tab);
  int* pick_e = tb;                                      // [64] expert of flat pick i
  float* pw = reinterpret_cast<float*>(tb + 64);         // [64] its weight
  int* sorted_e = tb + 128;                              // [64]
  int* sorted_tok = tb + 192;                            // [64] token of sorted row r
  int* inv = tb + 256;                                   // [64] sorted row of flat pick i
  int* act_e = tb + 320;                                 // [64] active experts, ascending
  int* act_row0 = tb + 384;                              // [64] first sorted row
  int* act_cnt = tb + 448;                               // [64]
  int* col_row = tb + 512;                               // [64 x 8] sorted row of (active expert, token) or -1
  int* hreq = tb + 1024;                                 // [64] h copy requested (control thread only)
  float* xscale = reinterpret_cast<float*>(tb + 1088);   // [8]
  int* misc = tb + 1096;                                 // [0] active, [1] items, [2..3] ballot counts
  unsigned* items = reinterpret_cast<unsigned*>(smem + a.o_items);
  float4* red = reinterpret_cast<float4*>(smem + a.o_red);
  float* dval = reinterpret_cast<float*>(smem + a.o_dval);
  uint64_t* fullb = reinterpret_cast<uint64_t*>(smem + a.o_bars);
  uint64_t* hbar = fullb + kFMaxSlots;

  if (tid == 0) {
    for (int s = 0; s < a.nslots; ++s) mbar_init(&fullb[s], 1);
    for (int j = 0; j < kFMaxR; ++j) mbar_init(&hbar[j], 1);
    fence_proxy_async();
  }
  if (tid < 64) hreq[tid] = 0;
  // token rows -> fp16 with a per-row power-of-two scale (one warp per row)
  if (warp < T) convert_rows_to_f16(a.hidden, a.act_dtype, xs, xscale, T, a.H, warp, kFWarps);
  {  // pair table: entry (byte, lane) = half2(code[hi nibble], code[lo nibble])
    const float code = c_nf4[lane & 15];
#pragma unroll 4
    for (int e = warp; e < 256; e += kFWarps) {
      const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
    }
  }

  // ---- routing -----------------------------------------------------------------------------
  const bool fused = a.router_w != nullptr;
  if (fused) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int cs = (int)cl.num_blocks(), cr = (int)cl.block_rank();
    float* logits = reinterpret_cast<float*>(smem + a.o_logits);
    const int tasks = a.E * ((T + kRouterTT - 1) / kRouterTT);
    const bool w16 = a.router_w_dtype != E4B_F32;
    for (int task = cr + cs * warp; task < tasks; task += cs * kFWarps) {
      if (w16)
        router_logits_warp16<8>(a.hidden, a.act_dtype, a.router_w, a.router_w_dtype, T, a.H, a.E, task % a.E,
                                (task / a.E) * kRouterTT, logits);
      else
        router_logits_warp(a.hidden, a.act_dtype, a.router_w, a.router_w_dtype, T, a.H, a.E, task % a.E,
                           (task / a.E) * kRouterTT, logits);
    }
    cl.sync();
    for (int i = tid; i < T * a.E; i += kFThreads) {  // the peers' logits into this CTA's copy
      const int t = i / a.E, e = i - t * a.E;
      const int owner = ((t / kRouterTT) * a.E + e) % cs;
      if (owner != cr) logits[i] = *cl.map_shared_rank(logits + i, owner);
    }
    cluster_arrive();  // matched by the wait before exit: peers keep their logits until all have read
    __syncthreads();
    if (warp < T) {
      int se = 0;
      float sw = 0.f;
      float* sv = reinterpret_cast<float*>(red) + warp * 64;
      int* si = reinterpret_cast<int*>(sv + 32);
#define E4B_FTOPK(EPL) router_topk_warp_ranked<EPL>(logits, T, a.E, k, a.route_kind, a.renorm, warp, sv, si, se, sw)
      if (a.E <= 32) E4B_FTOPK(1);
      else if (a.E <= 64) E4B_FTOPK(2);
      else if (a.E <= 128) E4B_FTOPK(4);
      else E4B_FTOPK(8);
#undef E4B_FTOPK
      if (lane < k) {
        pick_e[warp * k + lane] = se;
        pw[warp * k + lane] = sw;
        if (blockIdx.x == 0) {
          a.topk_idx_out[warp * k + lane] = se;
          a.topk_w_out[warp * k + lane] = sw;
        }
      }
    }
  } else if (tid < R) {
    pick_e[tid] = stack_expert(a.topk_idx[tid], a.emap, a.routed, a.E, a.err, blockIdx.x == 0);
    pw[tid] = load_as_f32(a.topk_w, a.w_dtype, tid);
  }
  __syncthreads();

  // ---- permutation: stable rank by (expert, flat index), as fast.py:126-133 -------------------
  if (tid < R) {
    const int e = pick_e[tid];
    int rank = 0;
    for (int j = 0; j < R; ++j) {
      const int ej = pick_e[j];
      rank += (ej < e) | ((ej == e) & (j < tid));
    }
    sorted_e[rank] = e;
    sorted_tok[rank] = tid / k;
    inv[tid] = rank;
  }
  __syncthreads();
  bool start = false;
  unsigned ball = 0;
  if (warp < kFMaxR / 32) {
    start = tid < R && (tid == 0 || sorted_e[tid - 1] != sorted_e[tid]);
    ball = __ballot_sync(0xffffffffu, start);
    if (lane == 0) misc[2 + warp] = __popc(ball);
  }
  __syncthreads();
  if (warp < kFMaxR / 32) {
    const int idx = (warp ? misc[2] : 0) + __popc(ball & ((1u << lane) - 1u));
    if (start) {
      act_e[idx] = sorted_e[tid];
      act_row0[idx] = tid;
    }
    if (tid == 0) misc[0] = misc[2] + misc[3];
  }
  for (int i = tid; i < kFMaxR * 8; i += kFThreads) col_row[i] = -1;
  __syncthreads();
  const int nact = misc[0];
  if (tid < nact) act_cnt[tid] = (tid + 1 < nact ? act_row0[tid + 1] : R) - act_row0[tid];
  int r0, r1;
  my_rows(a.H, r0, r1);
  const int nr = r1 - r0;
  const int tpe = n1 / 16;
  const int chH = (a.H + kFChunk - 1) / kFChunk, chI = (a.I + kFChunk - 1) / kFChunk;
  const int ntl = (nr + 15) / 16;
  __syncthreads();
  if (tid < R) {  // active index of each sorted row -> (expert, token) column map
    const int r = inv[tid];
    int j = 0;
    while (j + 1 < nact && act_row0[j + 1] <= r) ++j;
    col_row[j * 8 + tid / k] = r;
  }
  if (tid == 0) {  // this CTA's item list
    int n = 0;
    auto push_down = [&](int j) {
      for (int rt = 0; rt < ntl; ++rt)
        for (int c = 0; c < chI; ++c) items[n++] = item_word(true, j, rt, c);
    };
    for (int j = 0; j < nact; ++j) {
      const int64_t base = (int64_t)j * tpe;
      int64_t g = base + ((((int64_t)blockIdx.x - base) % G) + G) % G;
      for (; g < base + tpe; g += G)
        for (int c = 0; c < chH; ++c) items[n++] = item_word(false, j, (int)(g - base), c);
      if (j >= kFLag) push_down(j - kFLag);
    }
    for (int j = max(0, nact - kFLag); j < nact; ++j) push_down(j);
    misc[1] = n;
  }
  __syncthreads();
  const int nitems = misc[1];
  const int S = a.nslots;
  if (warp == 0)
    for (int n = 0; n < S && n < nitems; ++n) issue_item(a, items[n], ring + n * kFSlot, &fullb[n], act_e, r0, nr);

  // ---- the item stream -----------------------------------------------------------------------
  bool dead = false;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  uint4 bf[2][2];          // B fragments of this warp's two blocks (token rows or h rows)
  int bkey = -1;           // which (kind, expert, chunk) they hold
  int next_h = 0;          // control thread: next expert whose h to prefetch (down order) ...
  unsigned seen = 0;       // ... and its counter as last read (relaxed; consumed one item later)
  bool polled = false;
  for (int n = 0; n < nitems; ++n) {
    const Item it = item_of(items[n]);
    const int K = it.down ? a.I : a.H;
    const int nch = it.down ? chI : chH;
    const int nb = min(kFChunk, K - it.ch * kFChunk) / 64;
    char* slot = ring + (n % S) * kFSlot;
    if (it.ch == 0) acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    // B fragments: column gq = token gq (gate_up: its fp16 row; down: its h row for expert j)
    const int key = it.down ? (1 << 30) | (it.j << 8) | it.ch : it.ch;
    if (key != bkey) {
      if (it.down) {
        if (tid == 0) request_h(a, it.j, true, 0u, hreq, hbar, act_row0, act_cnt, hs);
        if (!mbar_wait(&hbar[it.j], 0)) {
          if (lane == 0) raise_error(a.err, E4B_ERR_TIMEOUT);
        }
      }
#pragma unroll
      for (int bi = 0; bi < 2; ++bi) {
        const int b = warp + 16 * bi;
        bf[bi][0] = bf[bi][1] = make_uint4(0, 0, 0, 0);
        if (b < nb && gq < T) {
          const __half* src = nullptr;
          if (!it.down) {
            src = xs + (int64_t)gq * a.H + it.ch * kFChunk + b * 64 + q * 16;
          } else {
            const int sr = col_row[it.j * 8 + gq];
            if (sr >= 0) src = hs + (int64_t)sr * a.hpitch + it.ch * kFChunk + b * 64 + q * 16;
          }
          if (src) {
            bf[bi][0] = *reinterpret_cast<const uint4*>(src);
            bf[bi][1] = *reinterpret_cast<const uint4*>(src + 8);
          }
        }
      }
      bkey = key;
    }
    if (!dead && !mbar_wait(&fullb[n % S], (n / S) & 1)) {
      raise_error(a.err, E4B_ERR_TIMEOUT);
      dead = true;
    }
    if (!dead) {
#pragma unroll
      for (int bi = 0; bi < 2; ++bi) {
        const int b = warp + 16 * bi;
        if (b < nb) {
          const uint2 wa = *reinterpret_cast<const uint2*>(slot + gq * kFPitch + b * 32 + q * 8);
          const uint2 wb = *reinterpret_cast<const uint2*>(slot + (gq + 8) * kFPitch + b * 32 + q * 8);
          const float sa = *reinterpret_cast<const float*>(slot + kFSlotW + gq * kFAPitch + b * 4);
          const float sb = *reinterpret_cast<const float*>(slot + kFSlotW + (gq + 8) * kFAPitch + b * 4);
          float pp[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t w0 = jj < 2 ? wa.x : wa.y, w1 = jj < 2 ? wb.x : wb.y;
            uint32_t a0, a1, a2, a3;
            if (jj & 1) {
              a0 = lut2<2>(lut, w0, lane4); a2 = lut2<3>(lut, w0, lane4);
              a1 = lut2<2>(lut, w1, lane4); a3 = lut2<3>(lut, w1, lane4);
            } else {
              a0 = lut2<0>(lut, w0, lane4); a2 = lut2<1>(lut, w0, lane4);
              a1 = lut2<0>(lut, w1, lane4); a3 = lut2<1>(lut, w1, lane4);
            }
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(&bf[bi][jj >> 1]);
            if (jj == 0)
              mma16816_zero(pp, a0, a1, a2, a3, xw[0], xw[1]);
            else
              mma16816(pp, a0, a1, a2, a3, xw[(jj & 1) * 2], xw[(jj & 1) * 2 + 1]);
          }
          acc[0] = fmaf(pp[0], sa, acc[0]);
          acc[1] = fmaf(pp[1], sa, acc[1]);
          acc[2] = fmaf(pp[2], sb, acc[2]);
          acc[3] = fmaf(pp[3], sb, acc[3]);
        }
      }
    }
    const bool last = it.ch == nch - 1;
    if (last) red[(n & 1) * kFThreads + warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    fence_proxy_async();  // generic reads of the slot before its refill by the async proxy
    dead = __syncthreads_or(dead);
    if (warp == 0 && !dead && n + S < nitems) issue_item(a, items[n + S], slot, &fullb[n % S], act_e, r0, nr);
    if (tid == 0) {  // prefetch the h of the next expert whose down tile comes, once it is ready
      while (next_h < nact && hreq[next_h]) {
        ++next_h;
        polled = false;
      }
      if (next_h < nact) {
        if (polled) request_h(a, next_h, false, seen, hreq, hbar, act_row0, act_cnt, hs);
        if (!hreq[next_h]) {  // read the counter now, look at the value after the next item
          seen = ld_relaxed_gpu(&a.sync[next_h]);
          polled = true;
        }
      }
    }
    if (last && warp == (n & (kFWarps - 1))) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < kFWarps; ++w) {  // fixed warp order
        const float4 v = red[(n & 1) * kFThreads + w * 32 + lane];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      const int c0 = act_row0[it.j], cn = act_cnt[it.j];
      if (!it.down) {
        // rows gq (gate / row) and gq + 8 (up / row + 8); columns 2q, 2q + 1 are tokens
        for (int r = c0; r < c0 + cn; ++r) {
          const int t = sorted_tok[r];
          if ((t >> 1) != q) continue;
          const float sc = xscale[t];
          const float va = ((t & 1) ? s.y : s.x) * sc, vb = ((t & 1) ? s.w : s.z) * sc;
          __half* hrow = a.h + (int64_t)r * a.I;
          if (a.has_gate) {
            hrow[8 * it.tile + gq] = store_cast<__half>(silu_f32(va) * vb, a.err);
          } else {
            hrow[16 * it.tile + gq] = store_cast<__half>(silu_f32(va), a.err);
            hrow[16 * it.tile + 8 + gq] = store_cast<__half>(silu_f32(vb), a.err);
          }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_gpu_add(&a.sync[it.j], 1u);
      } else {
        for (int r = c0; r < c0 + cn; ++r) {
          const int t = sorted_tok[r];
          if ((t >> 1) != q) continue;
          const int rl = 16 * it.tile + gq;
          if (rl < nr) dval[r * a.drows + rl] = (t & 1) ? s.y : s.x;
          if (rl + 8 < nr) dval[r * a.drows + rl + 8] = (t & 1) ? s.w : s.z;
        }
      }
    }
  }
  __syncthreads();

  // ---- combine: out[t, r] = sum over slots, in order, of down[inv[t*k+s], r] * w[t, s] -----------
  for (int i = tid; i < T * nr; i += kFThreads) {
    const int t = i / nr, rl = i - t * nr;
    float o = 0.f;
    for (int s = 0; s < k; ++s) o = fmaf(dval[inv[t * k + s] * a.drows + rl], pw[t * k + s], o);
    reinterpret_cast<OutT*>(a.out)[(int64_t)t * a.H + r0 + rl] = out_cast<OutT>(o, a.err);
  }

  // ---- drain, then the last CTA re-arms the counters for the next launch -------------------------
  if (tid == 0) {
    if (dead)
      for (int n = max(0, nitems - S); n < nitems; ++n) (void)mbar_wait(&fullb[n % S], (n / S) & 1);
    for (int j = 0; j < nact; ++j)
      if (hreq[j]) (void)mbar_wait(&hbar[j], 0);
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync[kFMaxR], 1u);
    if (prev == (unsigned)G - 1) {
      for (int j = 0; j < kFMaxR; ++j) a.sync[j] = 0u;
      a.sync[kFMaxR] = 0u;
      __threadfence();
    }
  }
  if (fused) cluster_wait();
}

struct FlowPlan {
  int nslots, o_ring, o_x, o_h, o_logits, o_tab, o_items, o_red, o_dval, o_bars, total, hpitch, drows;
};

static int round_up(int x, int a) { return (x + a - 1) / a * a; }

static bool flow_plan(const e4b_moe_desc& d, int grid, FlowPlan& p) {
  const int T = d.tokens, R = d.tokens * d.top_k;
  int o = kFLut;
  p.o_x = o;
  o = round_up(o + T * d.hidden * 2, 128);
  p.hpitch = d.intermediate + 8;
  p.o_h = o;
  o = round_up(o + R * p.hpitch * 2, 128);
  p.o_logits = o;
  o = round_up(o + T * d.num_experts * 4, 128);
  p.o_tab = o;
  o = round_up(o + kFTabInts * 4 + 256, 128);
  p.o_items = o;
  o = round_up(o + kFMaxItems * 4, 128);
  p.o_red = o;
  o = round_up(o + 2 * kFThreads * 16, 128);
  const int max_rows = (d.hidden + grid - 1) / grid;
  p.drows = round_up(max_rows, 16);
  p.o_dval = o;
  o = round_up(o + R * p.drows * 4, 128);
  p.o_bars = o;
  o = round_up(o + (kFMaxSlots + kFMaxR) * 8, 128);
  p.o_ring = o;
  const int slots = (kSmemCap - o) / kFSlot;
  p.nslots = slots > kFMaxSlots ? kFMaxSlots : slots;
  if (p.nslots < 3) return false;
  p.total = o + p.nslots * kFSlot;
  return true;
}

// Items one CTA can get: its gate_up tiles over all active experts plus its down tiles.
static int64_t flow_items_bound(const e4b_moe_desc& d, int grid) {
  const int64_t R = (int64_t)d.tokens * d.top_k;
  const int64_t nact = R < d.num_experts ? R : d.num_experts;
  const int64_t n1 = d.has_gate ? 2 * d.intermediate : d.intermediate;
  const int64_t tiles = nact * (n1 / 16);
  const int64_t chH = (d.hidden + kFChunk - 1) / kFChunk, chI = (d.intermediate + kFChunk - 1) / kFChunk;
  const int64_t rows = (d.hidden + grid - 1) / grid;
  // round-robin over the grid per expert: at most ceil(tiles_per_expert / grid) per expert
  const int64_t per_expert = (n1 / 16 + grid - 1) / grid;
  (void)tiles;
  return nact * per_expert * chH + nact * ((rows + 15) / 16) * chI;
}

struct DevInfo {
  int sms = 0;
  int cluster = 0;   // cluster size of the fused-router launch
  int grid_cl = 0;   // its grid
  bool configured[3] = {false, false, false};
};
std::mutex g_flow_mu;
DevInfo g_flow_dev[64];

static bool dev_info(DevInfo*& out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lk(g_flow_mu);
  DevInfo& di = g_flow_dev[dev];
  if (!di.sms && cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  out = &di;
  return di.sms > 0;
}

template <typename OutT>
static bool configure(DevInfo& di, int idx) {
  std::lock_guard<std::mutex> lk(g_flow_mu);
  if (di.configured[idx]) return true;
  auto kern = nf4_decode_flow_kernel<OutT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess) return false;
  if (!di.cluster) {  // largest grid of co-resident clusters, clusters of 4 or 2
    int best = 0, best_cs = 1;
    for (int cs : {4, 2}) {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(di.sms / cs * cs);
      cfg.blockDim = dim3(kFThreads);
      cfg.dynamicSmemBytes = kSmemCap;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = cs;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int ncl = 0;
      if (cudaOccupancyMaxActiveClusters(&ncl, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      if (ncl * cs > best) {
        best = ncl * cs;
        best_cs = cs;
      }
    }
    if (best <= 0) return false;
    di.cluster = best_cs;
    di.grid_cl = best > di.sms ? di.sms : best;
  }
  di.configured[idx] = true;
  return true;
}

}  // namespace

bool decode_flow_eligible(const e4b_moe_desc& d, bool fused_router) {
  if (decode_mode() != 1) return false;
  if (d.weight_format != E4B_FMT_NF4 || d.lora_rank != 0) return false;
  if (d.tokens < 1 || d.tokens > kFMaxT || (int64_t)d.tokens * d.top_k > kFMaxR) return false;
  if (d.hidden % 256 || d.intermediate % 256) return false;
  if (d.intermediate / 8 > 0xFFFF) return false;
  if (!is_act_dtype(d.act_dtype)) return false;
  if ((int64_t)d.num_experts * (d.has_gate ? 2 * d.intermediate : d.intermediate) >= (1ll << 31)) return false;
  if ((int64_t)d.num_experts * d.hidden >= (1ll << 31)) return false;
  if (fused_router && ((int64_t)d.tokens * d.num_experts > kFMaxLogits || d.num_experts > 256)) return false;
  DevInfo* di = nullptr;
  if (!dev_info(di)) return false;
  FlowPlan p;
  if (!flow_plan(d, di->sms, p)) return false;
  if (flow_items_bound(d, di->sms / 4 * 2) > kFMaxItems) return false;
  return true;
}

e4b_status launch_decode_flow(const e4b_moe_desc& d, const e4b_moe_tensors* t, void* h, void* sync, int* err,
                              cudaStream_t s, const DecodeRouter* router) {
  DevInfo* di = nullptr;
  if (!dev_info(di)) return E4B_ERR_CUDA;
  const int idx = d.out_dtype == E4B_BF16 ? 0 : d.out_dtype == E4B_F16 ? 1 : 2;
  bool ok = idx == 0 ? configure<__nv_bfloat16>(*di, idx) : idx == 1 ? configure<__half>(*di, idx)
                                                                      : configure<float>(*di, idx);
  if (!ok) return E4B_ERR_CUDA;
  const bool fused = router != nullptr;
  const int grid = fused ? di->grid_cl : di->sms;
  FlowPlan p;
  if (!flow_plan(d, grid, p)) return E4B_ERR_UNSUPPORTED;
  if (flow_items_bound(d, grid) > kFMaxItems) return E4B_ERR_UNSUPPORTED;
  FlowArgs a{};
  a.hidden = t->hidden;
  a.act_dtype = d.act_dtype;
  a.topk_idx = t->topk_idx;
  a.topk_w = t->topk_w;
  a.w_dtype = d.weight_dtype;
  a.emap = t->expert_map;
  a.routed = d.routed_experts;
  a.gu_packed = static_cast<const uint8_t*>(t->gate_up_packed);
  a.gu_absmax = static_cast<const float*>(t->gate_up_absmax);
  a.dn_packed = static_cast<const uint8_t*>(t->down_packed);
  a.dn_absmax = static_cast<const float*>(t->down_absmax);
  a.T = d.tokens;
  a.k = d.top_k;
  a.E = d.num_experts;
  a.H = d.hidden;
  a.I = d.intermediate;
  a.has_gate = d.has_gate;
  a.out = t->out;
  a.out_dtype = d.out_dtype;
  a.h = static_cast<__half*>(h);
  a.sync = static_cast<unsigned*>(sync);
  a.err = err;
  if (fused) {
    a.router_w = router->weight;
    a.router_w_dtype = router->weight_dtype;
    a.route_kind = router->kind;
    a.renorm = router->norm_topk_prob;
    a.topk_idx_out = router->topk_idx;
    a.topk_w_out = router->topk_w;
    a.w_dtype = E4B_F32;
  }
  a.nslots = p.nslots;
  a.o_ring = p.o_ring;
  a.o_x = p.o_x;
  a.o_h = p.o_h;
  a.o_logits = p.o_logits;
  a.o_tab = p.o_tab;
  a.o_items = p.o_items;
  a.o_red = p.o_red;
  a.o_dval = p.o_dval;
  a.o_bars = p.o_bars;
  a.hpitch = p.hpitch;
  a.drows = p.drows;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = p.total;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = fused ? di->cluster : 1;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = fused ? 1 : 0;
  cudaError_t e;
  switch (d.out_dtype) {
    case E4B_BF16: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<__nv_bfloat16>, a); break;
    case E4B_F16: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<__half>, a); break;
    default: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<float>, a); break;
  }
  return e == cudaSuccess ? E4B_OK : E4B_ERR_CUDA;
}

}  // namespace e4b
