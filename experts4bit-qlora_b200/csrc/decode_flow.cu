// Whole expert layer in one launch for the bs=1..8 decode regime (NF4, no
// adapters): router (optional) -> permute -> gate_up GEMV + SwiGLU -> down GEMV
// -> weighted combine, the per-layer chain of experts4bit_qlora/engines/fast.py:100-160.
//
// One CTA per SM, three roles after a common set-up:
//  * Set-up: the NF4 pair table, token rows to fp16; with the router fused, the
//    CTAs of a thread-block cluster split the (expert, token tile) logit tasks,
//    gather the peers' logits through distributed shared memory and run the same
//    ranked top-k (no grid-wide barrier); the stable permutation; the CTA's item
//    list. An item is 16 weight rows x up to 2048 K elements:
//      gate_up tile (8 gate + the 8 matching up rows of one expert), dealt
//        round-robin over the grid in expert-major order, so expert j's h is
//        complete at ~ (j + 1) / active of the gate_up phase;
//      down tile (the CTA's own output rows of one expert), placed two experts
//        after that expert's gate_up tiles.
//  * Producer warp: streams the items through a ring of shared-memory slots (two
//    swizzled TMA boxes of weights + two of absmax per item, mbarrier completion),
//    refilling a slot when the compute warps release it; meanwhile it polls the
//    tile counters of the experts whose down tiles come next and, once an expert's
//    gate_up tiles are all published, bulk-copies its h rows into shared memory.
//  * Compute warps (8): each takes every 8th 64-element K block of an item, with
//    the token / h fragments of its blocks in registers; NF4 codes decode through a
//    per-lane pair table (conflict-free LDS) into mma.sync m16n8k16 (fp32
//    accumulation), the block absmax folded in fp32 per block. A finished tile's
//    partial sums go to a reduction buffer.
//  * Epilogue warp: sums the 8 partials in warp order; gate_up: SwiGLU, h rows
//    (fp16) to global memory, a release increment of the expert's tile counter;
//    down: the rows stay in shared memory for the combine.
//  * Combine: each CTA owns whole output rows, so the fixed slot-order weighted sum
//    needs no further synchronisation.
// No role waits on another CTA except through the tile counters, and no CTA-wide
// barrier separates items. Counters live at a fixed offset of the workspace
// (kFlowSyncOffset), must be zero before the first launch and are zeroed again by
// the last CTA to finish. Every wait is bounded; a timeout raises E4B_ERR_TIMEOUT,
// records the wait in the workspace header (kFlowDiagWord) and the kernel runs to
// its end. Device errors go straight into the sticky workspace error word.
#include <cooperative_groups.h>

#include <mutex>

#include "convert.cuh"
#include "decode_layer.cuh"
#include "router.cuh"
#include "stream_core.cuh"
#include "tmap.cuh"

// Profiling instrumentation, compiled only with -DE4B_TRACE: thread 0 of every CTA stamps
// %globaltimer at the kernel's phase boundaries and at six points of every item.
#ifdef E4B_TRACE
__device__ unsigned long long g_flow_trace[160 * (8 + 64 * 6)];
extern "C" __attribute__((visibility("default"))) int e4b_flow_trace_read(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, g_flow_trace, n * sizeof(unsigned long long));
}
#define FT_K(i)                                                              \
  if (threadIdx.x == 0 && blockIdx.x < 160) {                                \
    unsigned long long t_;                                                   \
    if ((i) == 0)                                                            \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                \
    else                                                                     \
      t_ = (unsigned long long)clock64();                                    \
    g_flow_trace[blockIdx.x * (8 + 64 * 6) + (i)] = t_;                      \
    if ((i) == 0) g_flow_trace[blockIdx.x * (8 + 64 * 6) + 7] = (unsigned long long)clock64(); \
  }
#define FT_I(n, i)                                                           \
  if (threadIdx.x == 0 && blockIdx.x < 160 && (n) < 64) {                    \
    g_flow_trace[blockIdx.x * (8 + 64 * 6) + 8 + (n) * 6 + (i)] = (unsigned long long)clock64(); \
  }
#else
#define FT_K(i)
#define FT_I(n, i)
#endif

namespace e4b {

namespace {

using stream::lut2;
using stream::mma16816;
using stream::mma16816_zero;

constexpr int kFWarps = 16;                  // compute warps: each takes every 16th K block of an item
constexpr int kFProducer = kFWarps;          // warp: TMA issue of the items
constexpr int kFEpilogue = kFWarps + 1;      // warp: partial-tile reduction, h / down-row stores
constexpr int kFFetch = kFWarps + 2;         // warp: tile-counter polls, h copies
constexpr int kFAll = kFWarps + 3;
constexpr int kFThreads = kFAll * 32;
constexpr int kFNR = 4;                      // partial-tile buffers between compute and epilogue
constexpr int kFBlk = 32 / kFWarps;          // K blocks per compute warp in a full 2048-element chunk
constexpr int kFChunk = 2048;               // K elements per item
// A slot holds one item as four TMA boxes: two weight boxes of 8 rows x up to 8 lines of 128 B
// ([line][row][128 B], 128-byte swizzle: row r's 16-byte units XOR r, conflict-free fragment reads)
// and their two absmax boxes of 8 rows x up to 32 floats (swizzled by the row width).
constexpr int kFWBox = 8 * 1024;
constexpr int kFABox = 32 * 8 * 4;
constexpr int kFSlot = 2 * kFWBox + 2 * kFABox;  // 18432 B, a multiple of 1024
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
  int* diag;            // first timed-out wait: [0] taken, [1] site, [2] CTA, [3] item / expert, [4] value
  uint32_t spins;       // bound of every wait (polls)
  const void* router_w;  // fused router when non-null
  int router_w_dtype, route_kind, renorm;
  int64_t* topk_idx_out;
  float* topk_w_out;
  // shared-memory plan (bytes), computed on the host
  int nslots, o_ring, o_x, o_h, o_logits, o_tab, o_items, o_red, o_dval, o_bars;
  int hpitch;           // halves per staged h row
  int drows;            // rows per pick in dval (the CTA's output rows, rounded up to 16)
};

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
// Programmatic dependent launch: this grid's CTAs may start while the previous kernel on the
// stream drains; everything that reads or writes memory another kernel touches waits here.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Records the first wait of the launch that gave up (site 1: weight copies of item `what`; 2: the
// tile counter of active expert `what`, `value` = the count seen; 3: the h copy of expert `what`;
// 4: a ring slot to refill (item `what`); 5: partial tiles to reduce; 6: a reduction buffer).
__device__ __forceinline__ void note_timeout(const FlowArgs& a, int site, int what, unsigned value) {
  raise_error(a.err, E4B_ERR_TIMEOUT);
  if (a.diag && atomicCAS(&a.diag[0], 0, 1) == 0) {
    a.diag[1] = site;
    a.diag[2] = blockIdx.x;
    a.diag[3] = what;
    a.diag[4] = (int)value;
  }
}

// One poll of a barrier phase that suspends at most about a microsecond (explicit suspend-time
// hint), so a bound in polls is a bound in time: kMaxSpins polls are a few seconds.
__device__ __forceinline__ bool try_wait_1us(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t spins) {
  for (uint32_t i = 0; i < spins; ++i)
    if (try_wait_1us(bar, parity)) return true;
  return false;
}

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

__host__ __device__ constexpr int box_lines_of(int kc) { return kc / 256 < 8 ? kc / 256 : 8; }
__host__ __device__ constexpr int abox_of(int kc) { return kc / 64 < 32 ? kc / 64 : 32; }

// Byte offset of lane (row r of a box, quad lane q)'s 8-byte piece of block bc in a weight box at a
// 1024-aligned shared address: line bc / 4 holds blocks 4 (bc / 4) .. +3; the swizzle XORs unit with r.
__device__ __forceinline__ int wpiece(int r, int q, int bc) {
  const int unit = (((bc & 3) << 1) | (q >> 1)) ^ r;
  return (bc >> 2) * 1024 + r * 128 + (unit << 4) + ((q & 1) << 3);
}
// Byte offset of (row r, block b) in an absmax box whose rows are S = 4 * floats bytes (16..128),
// stored with the S-byte swizzle (none for 16 B).
__device__ __forceinline__ int apiece(int r, int b, int S) {
  return r * S + ((((b >> 2) ^ ((r * S) >> 7)) & (S / 16 - 1)) << 4) + ((b & 3) << 2);
}

// One item into its slot (one thread): the two 8-row weight boxes and their absmax boxes. A down
// tile's second box may reach rows of the next CTA's range (read, not used) or past the stack
// (zero-filled by the TMA unit).
__device__ __forceinline__ void issue_item(const FlowArgs& a, unsigned w, char* slot, uint64_t* bar,
                                           const int* act_e, int r0, const CUtensorMap* wgu, const CUtensorMap* agu,
                                           const CUtensorMap* wdn, const CUtensorMap* adn) {
  const Item it = item_of(w);
  const int e = act_e[it.j];
  const int K = it.down ? a.I : a.H;
  // the boxes are as wide as a full chunk of this projection (K < 2048: all of K); a last, shorter
  // chunk reads past the row end, which the TMA unit zero-fills and still counts
  const uint32_t wbytes = box_lines_of(K) * 1024, abytes = abox_of(K) * 32;
  const CUtensorMap* wm = it.down ? wdn : wgu;
  const CUtensorMap* am = it.down ? adn : agu;
  mbar_arrive_expect_tx(bar, 2 * (wbytes + abytes));
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    int row;
    if (it.down) {
      row = e * a.H + r0 + 16 * it.tile + 8 * h;
    } else {
      const int n1 = a.has_gate ? 2 * a.I : a.I;
      row = a.has_gate ? e * n1 + (h == 0 ? 8 * it.tile : a.I + 8 * it.tile) : e * n1 + 16 * it.tile + 8 * h;
    }
    tma_load_3d(slot + h * kFWBox, wm, 0, row, it.ch * (kFChunk / 256), bar);
    tma_load_2d(slot + 2 * kFWBox + h * kFABox, am, it.ch * (kFChunk / 64), row, bar);
  }
}

template <typename OutT>
__global__ void __launch_bounds__(kFThreads, 1)
    nf4_decode_flow_kernel(const FlowArgs a, const __grid_constant__ CUtensorMap wgu,
                           const __grid_constant__ CUtensorMap agu, const __grid_constant__ CUtensorMap wdn,
                           const __grid_constant__ CUtensorMap adn) {
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
  int* hreq = tb + 1024;                                 // [64] h copy requested (fetch warp)
  float* xscale = reinterpret_cast<float*>(tb + 1088);   // [8]
  int* misc = tb + 1096;                                 // [0] active, [1] items, [2..3] ballot counts, [4] issued
  unsigned* items = reinterpret_cast<unsigned*>(smem + a.o_items);
  float4* red = reinterpret_cast<float4*>(smem + a.o_red);
  float* dval = reinterpret_cast<float*>(smem + a.o_dval);
  uint64_t* fullb = reinterpret_cast<uint64_t*>(smem + a.o_bars);  // [slot] item landed
  uint64_t* emptyb = fullb + kFMaxSlots;                            // [slot] compute warps done with it
  uint64_t* redfull = emptyb + kFMaxSlots;                          // [buffer] partials written
  uint64_t* redfree = redfull + kFNR;                               // [buffer] partials reduced
  uint64_t* hbar = redfree + kFNR;                                  // [active expert] h rows landed

  // ---- prologue: nothing here touches memory that another kernel writes ----------------------
  FT_K(0);
  launch_dependents();  // the next layer's grid may be scheduled as this one's CTAs finish
  if (tid < 4) {        // descriptors into the TMA unit's cache before the first copies
    const CUtensorMap* m = tid == 0 ? &wgu : tid == 1 ? &agu : tid == 2 ? &wdn : &adn;
    asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
  }
  if (tid < kFMaxSlots) {
    mbar_init(&fullb[tid], 1);
    mbar_init(&emptyb[tid], kFWarps);
  }
  if (tid < kFNR) {
    mbar_init(&redfull[tid], kFWarps);
    mbar_init(&redfree[tid], 1);
  }
  if (tid < kFMaxR) {
    mbar_init(&hbar[tid], 1);
    hreq[tid] = 0;
  }
  if (tid == 0) misc[4] = 0;
  fence_proxy_async();
  if (a.router_w && tid == 32) {  // this CTA's share of the router weights (parameters) into L2
    const int wb = a.router_w_dtype == E4B_F32 ? 4 : 2;
    const int64_t bytes = (int64_t)a.E * a.H * wb;
    const int64_t part = ((bytes / gridDim.x) + 15) / 16 * 16;
    const int64_t off = part * blockIdx.x;
    if (off < bytes) prefetch_l2(static_cast<const char*>(a.router_w) + off, (uint32_t)min(part, bytes - off));
  }
  {  // pair table: entry (byte, lane) = half2(code[hi nibble], code[lo nibble])
    const float code = c_nf4[lane & 15];
#pragma unroll 4
    for (int e = warp; e < 256; e += kFAll) {
      const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
    }
  }
  grid_dependency_wait();
  FT_K(1);
  // token rows -> fp16 with a per-row power-of-two scale (one warp per row)
  if (warp < T) convert_rows_to_f16(a.hidden, a.act_dtype, xs, xscale, T, a.H, warp, kFAll);

  // ---- routing -----------------------------------------------------------------------------
  const bool fused = a.router_w != nullptr;
  if (fused) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int cs = (int)cl.num_blocks(), cr = (int)cl.block_rank();
    float* logits = reinterpret_cast<float*>(smem + a.o_logits);
    const int tasks = a.E * ((T + kRouterTT - 1) / kRouterTT);
    const bool w16 = a.router_w_dtype != E4B_F32;
    for (int task = cr + cs * warp; task < tasks; task += cs * kFAll) {
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
  } else if (tid >= kFProducer * 32 && tid - kFProducer * 32 < R) {  // warps 8-9: their loads beside the rows'
    const int i = tid - kFProducer * 32;
    pick_e[i] = stack_expert(a.topk_idx[i], a.emap, a.routed, a.E, a.err, blockIdx.x == 0);
    pw[i] = load_as_f32(a.topk_w, a.w_dtype, i);
  }
  __syncthreads();

  FT_K(2);
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
    int first = blockIdx.x;  // this CTA's first tile of expert j: tiles are dealt round-robin over the grid
    for (int j = 0; j < nact; ++j) {
      int tt = first;
      for (; tt < tpe; tt += G)
        for (int c = 0; c < chH; ++c) items[n++] = item_word(false, j, tt, c);
      first = tt - tpe;  // the next expert continues the deal where this one stopped
      if (j >= kFLag) push_down(j - kFLag);
    }
    for (int j = max(0, nact - kFLag); j < nact; ++j) push_down(j);
    misc[1] = n;
  }
  __syncthreads();
  const int nitems = misc[1];
  const int S = a.nslots;
  FT_K(3);
  const unsigned need = (unsigned)(n1 / 16);  // gate_up tiles of an expert
  bool dead = false;

  if (warp == kFProducer) {
    // ---- producer: items into the ring as the compute warps release slots -----------------------
    if (lane == 0) {
      for (int n = 0; n < nitems && !dead; ++n) {
        const int s_ = n % S;
        if (n >= S && !wait_bar(&emptyb[s_], ((n / S) - 1) & 1, a.spins)) {
          note_timeout(a, 4, n, 0);
          dead = true;
          break;
        }
        issue_item(a, items[n], ring + s_ * kFSlot, &fullb[s_], act_e, r0, &wgu, &agu, &wdn, &adn);
        misc[4] = n + 1;  // items issued (the drain waits for these only)
      }
    }
  } else if (warp == kFFetch) {
    // ---- fetch: h rows of each expert, in down order, once its gate_up tiles are all published -------
    if (lane == 0 && nr > 0) {
      int j = 0;
      for (uint32_t i = 0; i < a.spins && j < nact; ++i) {
        if (ld_relaxed_gpu(&a.sync[j]) < need) {
          __nanosleep(64);
          continue;
        }
        fence_acq_rel_gpu();          // the relaxed observation becomes an acquire
        fence_proxy_async_global();   // the acquired h stores, before the async-proxy reads
        const int cnt = act_cnt[j], row0 = act_row0[j];
        mbar_arrive_expect_tx(&hbar[j], (uint32_t)(cnt * a.I * 2));
        for (int c = 0; c < cnt; ++c)
          bulk_g2s(hs + (int64_t)(row0 + c) * a.hpitch, a.h + (int64_t)(row0 + c) * a.I, (uint32_t)(a.I * 2),
                   &hbar[j]);
        hreq[j] = 1;
        ++j;
      }
      for (; j < nact; ++j) {  // gave up: complete the barriers without data
        note_timeout(a, 2, j, ld_relaxed_gpu(&a.sync[j]));
        hreq[j] = 1;
        mbar_arrive(&hbar[j]);
      }
    }
  } else if (warp == kFEpilogue) {
    // ---- epilogue: reduce each tile's partials in fixed warp order, publish h / keep down rows ----
    int t = 0;
    for (int n = 0; n < nitems; ++n) {
      const Item it = item_of(items[n]);
      if (it.ch != (it.down ? chI : chH) - 1) continue;
      const int rb = t % kFNR;
      if (!wait_bar(&redfull[rb], (t / kFNR) & 1, a.spins)) {
        if (lane == 0) note_timeout(a, 5, n, 0);
        break;
      }
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < kFWarps; ++w) {
        const float4 v = red[rb * kFWarps * 32 + w * 32 + lane];
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&redfree[rb]);  // the buffer is read: the compute warps may refill it
      ++t;
      const int c0 = act_row0[it.j], cn = act_cnt[it.j];
      if (!it.down) {
        // rows gq (gate / row) and gq + 8 (up / row + 8); columns 2q, 2q + 1 are tokens
        for (int r = c0; r < c0 + cn; ++r) {
          const int tk = sorted_tok[r];
          if ((tk >> 1) != q) continue;
          const float sc = xscale[tk];
          const float va = ((tk & 1) ? sum.y : sum.x) * sc, vb = ((tk & 1) ? sum.w : sum.z) * sc;
          __half* hrow = a.h + (int64_t)r * a.I;
          if (a.has_gate) {
            hrow[8 * it.tile + gq] = store_cast<__half>(silu_f32(va) * vb, a.err);
          } else {
            hrow[16 * it.tile + gq] = store_cast<__half>(silu_f32(va), a.err);
            hrow[16 * it.tile + 8 + gq] = store_cast<__half>(silu_f32(vb), a.err);
          }
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          red_release_gpu_add(&a.sync[it.j], 1u);
        }
      } else {
        for (int r = c0; r < c0 + cn; ++r) {
          const int tk = sorted_tok[r];
          if ((tk >> 1) != q) continue;
          const int rl = 16 * it.tile + gq;
          if (rl < nr) dval[r * a.drows + rl] = (tk & 1) ? sum.y : sum.x;
          if (rl + 8 < nr) dval[r * a.drows + rl + 8] = (tk & 1) ? sum.w : sum.z;
        }
      }
    }
  } else {
    // ---- compute warps: every 8th K block of each item, partial tiles to the epilogue -------------
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    uint4 bf[kFBlk][2];  // B fragments of this warp's blocks (token rows or h rows)
    int bkey = -1;   // which (kind, expert, chunk) they hold
    int t = 0;       // finished tiles
    for (int n = 0; n < nitems; ++n) {
      FT_I(n, 0);
      const Item it = item_of(items[n]);
      const int K = it.down ? a.I : a.H;
      const int nch = it.down ? chI : chH;
      const int nb = min(kFChunk, K - it.ch * kFChunk) / 64;
      const int arow = abox_of(K) * 4;  // bytes per absmax box row
      const int s_ = n % S;
      const char* slot = ring + s_ * kFSlot;
      if (it.ch == 0) acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
      // B fragments: column gq = token gq (gate_up: its fp16 row; down: its h row for expert j)
      const int key = it.down ? (1 << 30) | (it.j << 8) | it.ch : it.ch;
      if (key != bkey) {
        if (it.down && !dead && !wait_bar(&hbar[it.j], 0, a.spins)) {
          if (lane == 0) note_timeout(a, 3, it.j, 0);
          dead = true;
        }
#pragma unroll
        for (int bi = 0; bi < kFBlk; ++bi) {
          const int b = warp + kFWarps * bi;
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
      FT_I(n, 1);
      if (!dead && !wait_bar(&fullb[s_], (n / S) & 1, a.spins)) {
        if (lane == 0) note_timeout(a, 1, n, 0);
        dead = true;
      }
      FT_I(n, 2);
      if (!dead) {
#pragma unroll
        for (int bi = 0; bi < kFBlk; ++bi) {
          const int b = warp + kFWarps * bi;
          if (b < nb) {
            const uint2 wa = *reinterpret_cast<const uint2*>(slot + wpiece(gq, q, b));
            const uint2 wb = *reinterpret_cast<const uint2*>(slot + kFWBox + wpiece(gq, q, b));
            const float sa = *reinterpret_cast<const float*>(slot + 2 * kFWBox + apiece(gq, b, arow));
            const float sb = *reinterpret_cast<const float*>(slot + 2 * kFWBox + kFABox + apiece(gq, b, arow));
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
      FT_I(n, 3);
      fence_proxy_async();  // this warp's reads of the slot, before its refill by the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&emptyb[s_]);
      if (it.ch == nch - 1) {  // the tile's partial sums to a reduction buffer
        const int rb = t % kFNR;
        if (t >= kFNR && !dead && !wait_bar(&redfree[rb], ((t / kFNR) - 1) & 1, a.spins)) {
          if (lane == 0) note_timeout(a, 6, n, 0);
          dead = true;
        }
        red[rb * kFWarps * 32 + warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&redfull[rb]);
        ++t;
      }
      FT_I(n, 4);
    }
  }
  FT_K(4);
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
    // every copy still in flight lands before the CTA exits: the ring's last S items and the h rows
    const int issued = misc[4];
    for (int n = max(0, issued - S); n < issued; ++n) (void)wait_bar(&fullb[n % S], (n / S) & 1, a.spins);
    for (int j = 0; j < nact; ++j)
      if (hreq[j]) (void)wait_bar(&hbar[j], 0, a.spins);
    __threadfence();
    const unsigned prev = atomicAdd(&a.sync[kFMaxR], 1u);
    if (prev == (unsigned)G - 1) {
      for (int j = 0; j < kFMaxR; ++j) a.sync[j] = 0u;
      a.sync[kFMaxR] = 0u;
      __threadfence();
    }
  }
  FT_K(5);
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
  o = round_up(o + kFNR * kFWarps * 32 * 16, 128);
  const int max_rows = (d.hidden + grid - 1) / grid;
  p.drows = round_up(max_rows, 16);
  p.o_dval = o;
  o = round_up(o + R * p.drows * 4, 128);
  p.o_bars = o;
  o = round_up(o + (2 * kFMaxSlots + 2 * kFNR + kFMaxR) * 8, 128);
  o = round_up(o, 1024);  // the swizzled boxes follow the shared address: 1024-aligned slots
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

// Bound of every wait of the flow kernel, in polls (E4B_FLOW_SPINS overrides, for diagnosis).
uint32_t flow_spins() {
  static const uint32_t v = [] {
    const char* e = getenv("E4B_FLOW_SPINS");
    const long n = e ? atol(e) : 0;
    return n > 0 ? (uint32_t)n : kMaxSpins;
  }();
  return v;
}

// E4B_FLOW_PDL=0 launches without programmatic dependent launch (A/B timing).
bool flow_pdl() {
  static const int v = [] {
    const char* e = getenv("E4B_FLOW_PDL");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return v != 0;
}

}  // namespace

bool decode_flow_eligible(const e4b_moe_desc& d, bool fused_router) {
  if (decode_mode() != 1) return false;
  if (d.weight_format != E4B_FMT_NF4 || d.lora_rank != 0) return false;
  if (d.tokens < 1 || d.tokens > kFMaxT || (int64_t)d.tokens * d.top_k > kFMaxR) return false;
  if (d.hidden % 256 || d.intermediate % 256) return false;
  // absmax boxes of 4, 8, 16 or 32 floats (a power of two under the box swizzle)
  for (int K : {d.hidden, d.intermediate})
    if (K < 2048 && (K & (K - 1))) return false;
  if (d.intermediate / 8 > 0xFFFF) return false;
  if (!encode_tiled_fn()) return false;
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
  a.diag = err + kFlowDiagWord;
  a.spins = flow_spins();
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
  cudaLaunchAttribute at[2];
  int na = 0;
  if (flow_pdl()) {  // programmatic dependent launch (the kernel waits before touching shared memory)
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (fused) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = di->cluster;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  // packed bytes as [lines (K/256)][rows][128 B]: a box of 8 rows x up to 8 lines lands row-major per
  // line, 128-byte swizzled; absmax as [rows][K/64] floats in boxes of 8 rows x up to 32 floats
  auto maps = [&](CUtensorMap& w, CUtensorMap& am, const void* packed, const void* absmax, int64_t rows, int K) {
    const cuuint64_t wdims[3] = {128, (cuuint64_t)rows, (cuuint64_t)(K / 256)};
    const cuuint64_t wstr[2] = {(cuuint64_t)(K / 2), 128};
    const cuuint32_t wbox[3] = {128, 8, (cuuint32_t)box_lines_of(K)};
    const cuuint64_t adims[2] = {(cuuint64_t)(K / 64), (cuuint64_t)rows};
    const cuuint64_t astr[1] = {(cuuint64_t)(K / 64) * 4};
    const cuuint32_t abox[2] = {(cuuint32_t)abox_of(K), 8};
    const int S = abox_of(K) * 4;
    const CUtensorMapSwizzle asw = S == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : S == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : S == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
    return encode_tiled(&w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, wdims, wstr, wbox, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_tiled(&am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, absmax, adims, astr, abox, asw);
  };
  CUtensorMap wgu, agu, wdn, adn;
  const int n1 = d.has_gate ? 2 * d.intermediate : d.intermediate;
  if (!maps(wgu, agu, t->gate_up_packed, t->gate_up_absmax, (int64_t)d.num_experts * n1, d.hidden) ||
      !maps(wdn, adn, t->down_packed, t->down_absmax, (int64_t)d.num_experts * d.hidden, d.intermediate))
    return E4B_ERR_CUDA;
  cudaError_t e;
  switch (d.out_dtype) {
    case E4B_BF16: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<__nv_bfloat16>, a, wgu, agu, wdn, adn); break;
    case E4B_F16: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<__half>, a, wgu, agu, wdn, adn); break;
    default: e = cudaLaunchKernelEx(&cfg, nf4_decode_flow_kernel<float>, a, wgu, agu, wdn, adn); break;
  }
  return e == cudaSuccess ? E4B_OK : E4B_ERR_CUDA;
}

}  // namespace e4b
