// Whole expert layer in one persistent launch for the decode regime (NF4, at
// most 128 picks, no adapters): the per-layer kernel chain of fast.py:100-160 --
// permute, grouped gate_up GEMM + SwiGLU, grouped down GEMM, weighted combine --
// as phases of one cooperative kernel with one CTA per SM:
//   phase 0  every CTA rebuilds the (at most 128-pick) stable expert-major
//            permutation in shared memory from top_k_index and starts its first
//            weight copies at once; meanwhile it converts the token rows (loaded
//            into registers at entry) to fp16 with a per-row power-of-two scale and
//            builds the NF4 pair table;
//   phase A  gate_up tiles: a warp pair owns 16 weight rows (8 gate + the 8
//            matching up rows) and streams them in items of up to 2048 K elements,
//            one 8 KB TMA box per 8 rows and one absmax box; fragments go to
//            mma.sync m16n8k16 with the tokens as the n8 operand; h rows (fp16) to
//            the workspace; each pair then starts its first down-weight copy,
//            which overlaps the barrier;                         grid barrier;
//   phase B  down tiles, activations (h) staged from L2;        grid barrier;
//   phase C  fixed-slot-order combine into the output.
// The arithmetic is the streaming GEMV's (gemv_stream.cu) and the combine
// kernel's, so the result equals the multi-kernel path bit for bit. Copy waits
// are bounded (a timeout raises E4B_ERR_TIMEOUT and the kernel runs to its end);
// the grid barriers are cooperative-launch grid syncs that every CTA reaches.
// Errors are collected per CTA and folded into the workspace's (sticky) error word
// by CTA 0 after the last barrier.
#include <cooperative_groups.h>

#include <atomic>
#include <mutex>
#include <new>

#include "convert.cuh"
#include "decode_layer.cuh"
#include "router.cuh"
#include "stream_core.cuh"
#include "tmap.cuh"
#include "nf4_prmt.cuh"

// Profiling instrumentation, compiled only with -DE4B_TRACE: per-CTA %globaltimer
// stamps at phase boundaries, read back with e4b_decode_trace_read.
#ifdef E4B_TRACE
__device__ unsigned long long g_dl_trace[1024 * 24];
extern "C" __attribute__((visibility("default"))) int e4b_decode_trace_read(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, g_dl_trace, n * sizeof(unsigned long long));
}
__device__ unsigned long long g_dl_pair[1024 * 8 * 4];  // per pair: phase A item0 ready, A done, B item0, B done
extern "C" __attribute__((visibility("default"))) int e4b_decode_pair_read(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, g_dl_pair, n * sizeof(unsigned long long));
}
#define DTRACE(i)                                                  \
  if (threadIdx.x == 0) {                                          \
    unsigned long long t_;                                         \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));        \
    g_dl_trace[blockIdx.x * 24 + (i)] = t_;                        \
  }
#define PTRACE(i)                                                  \
  if (lane == 0 && member == 0) {                                  \
    unsigned long long t_;                                         \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));        \
    g_dl_pair[(blockIdx.x * 8 + pair) * 4 + (i)] = t_;             \
  }
// slice kernel: per CTA 32 stamps (stage waits and releases of warps 1 and 15, refills by thread 0)
#define STRACE(w, i)                                               \
  if (warp == (w) && lane == 0 && (i) < 32) {                      \
    unsigned long long t_;                                         \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));        \
    g_dl_pair[blockIdx.x * 32 + (i)] = t_;                         \
  }
#else
#define DTRACE(i)
#define PTRACE(i)
#define STRACE(w, i)
#endif

namespace e4b {

namespace {

using stream::kLut;
using stream::kPairs;
using stream::kThreads;
using stream::kWarps;
using stream::lut2;
using stream::mma16816;
using stream::mma16816_zero;
using stream::named_barrier;

constexpr int kMaxPicks = 128;
constexpr int kMaxLogits = 4096;          // T x E of the fused router, in shared memory
// One item per tile up to K = 2048: the pair-table lookups, not the copies, bound an item, so
// splitting tiles into smaller items in flight together does not pay here.
constexpr int kDChunk = 2048;             // K elements per item
constexpr int kDSlots = 1;                // items in flight per pair
constexpr int kWBoxCap = 8 * 1024;        // one 8-row group, up to 8 lines of 128 B
constexpr int kABoxCap = 32 * 8 * 4;      // one 8-row group, up to 32 absmax floats
constexpr int kDSlotBytes = 2 * kWBoxCap + 2 * kABoxCap;  // 18 KB, a multiple of 1024
constexpr int kDXBudget = 20 * 1024;      // token rows (then h rows) staged in shared memory

__host__ __device__ constexpr int box_lines(int K) { return K / 256 < 8 ? K / 256 : 8; }
__host__ __device__ constexpr int abox_floats(int K) { return K / 64 < 32 ? K / 64 : 32; }

// Byte offset of (row r, block b) in an absmax box whose rows are S = abox_floats * 4 bytes
// (16..128), stored with the S-byte swizzle (none for 16): the 16-byte unit of block b is XORed
// with address bits 7.. of the row, which spreads the 8 rows over distinct banks.
__device__ __forceinline__ int aofs(int r, int b, int S) {
  return r * S + ((((b >> 2) ^ ((r * S) >> 7)) & (S / 16 - 1)) << 4) + ((b & 3) << 2);
}

struct DSmem {
  static constexpr int lut = 0;
  static constexpr int x = kLut;
  static constexpr int slots = x + kDXBudget;
  static constexpr int red = slots + kPairs * kDSlots * kDSlotBytes;
  static constexpr int bars = red + kPairs * 32 * 8 * 4;
  static constexpr int tables = bars + kPairs * kDSlots * 8;
  // int tables of kMaxPicks: pick expert, sorted expert, sorted token, inverse, active expert/row0/count;
  // 16 token scales, 16 misc words, kMaxPicks top-k weights, 16 row maxima
  static constexpr int logits = tables + 7 * kMaxPicks * 4 + 16 * 4 + 16 * 4 + kMaxPicks * 4 + 16 * 4;
  static constexpr int total = logits + kMaxLogits * 4;  // fused router: [T, E] fp32
};
static_assert(DSmem::slots % 1024 == 0 && kDSlotBytes % 1024 == 0, "swizzled boxes need 1024-byte alignment");
static_assert(DSmem::total <= 232448, "shared memory budget");
static_assert(16 * 64 * 4 <= kPairs * 32 * 8 * 4, "top-k selection slots of 16 token warps fit the reduction area");

struct DecodeArgs {
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
  __half* h;                   // [R, I]
  __half* down_rows;           // [R, H]
  int* cta_err;                // [gridDim.x]
  int* err;
  // fused router (router_w != null): logits of x . W_r^T and the top-k replace topk_idx / topk_w
  const void* router_w;
  int router_w_dtype, route_kind, renorm;
  int64_t* topk_idx_out;       // [T, k] (written by CTA 0)
  float* topk_w_out;           // [T, k]
  float* router_logits;        // [T, E] global scratch: logits spread over the grid, then a grid sync
  float* part;                 // slice kernel: fp32 partial down rows [R][I / 64][H]
  int slice_flags;             // slice kernel stage hand-off: bit 0 no per-warp proxy fence before a
                               // release, bit 1 the last warp to release a stage issues its refill
  int cluster;                 // > 1: launched in clusters of this size; the router's tasks are split
                               // over the cluster and the logits exchanged through distributed shared
                               // memory (router_logits unused)
};

struct Tables {
  int* pick_e;     // expert of flat pick i
  int* sorted_e;   // expert of sorted row r
  int* sorted_tok; // token of sorted row r
  int* inv;        // sorted row of flat pick i
  int* act_e;
  int* act_row0;
  int* act_cnt;
  float* xscale;   // per token row
  float* w;        // top-k weight of flat pick i (fp32)
  unsigned* rowmax;// per token row: max |x| as float bits
  int* misc;       // [0] active experts, [1] CTA error, [2..5] warp start counts, [7] error fold
};

__device__ __forceinline__ void cta_raise(int* cta_err, int code) { atomicCAS(cta_err, 0, code); }

template <typename T> __device__ __forceinline__ T store_cast_out(float v, int*) { return from_f32<T>(v); }
template <> __device__ __forceinline__ __half store_cast_out<__half>(float v, int* err) {
  return store_cast<__half>(v, err);
}

// Eight 16-bit activations (bf16 or fp16) -> fp32.
__device__ __forceinline__ void unpack8(const uint4& r, int dtype, float (&v)[8]) {
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

struct Phase {
  const CUtensorMap* wmap;
  const CUtensorMap* amap;
  int N, K, epilogue, tiles_per_expert;
  const __half* x;     // token rows: shared memory (phase A) or global (phase B)
  int xpitch;          // halves
  bool x_mapped;       // sorted row -> token row through sorted_tok, and per-token scales
  __half* out;
  int Nout;
};

__device__ __forceinline__ int phase_chunks(const Phase& p) { return (p.K + kDChunk - 1) / kDChunk; }

// The pair's items: tiles gp, gp + npairs, ... below nact * tiles_per_expert, chunks each.
__device__ __forceinline__ int phase_items(const Phase& p, int nact, int gp) {
  const int npairs = gridDim.x * kPairs;
  const int limit = nact * p.tiles_per_expert;
  return (limit > gp ? (limit - gp + npairs - 1) / npairs : 0) * phase_chunks(p);
}

__device__ __forceinline__ int group_row(const Phase& p, int tile, int h) {
  if (p.epilogue == E4B_EPI_SWIGLU) return h == 0 ? tile * 8 : (p.N >> 1) + tile * 8;
  return tile * 16 + 8 * h;
}

// Copies of the pair's item n (of this phase; n0 items before it) into ring slot (n0 + n) % kDSlots
// (pair leader only).
__device__ __forceinline__ void issue_item(const Phase& p, const Tables& tb, char* smem, int gp, int n, int n0) {
  const int pair = gp - blockIdx.x * kPairs;
  char* slot = smem + DSmem::slots + (pair * kDSlots + (n0 + n) % kDSlots) * kDSlotBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + DSmem::bars) + pair * kDSlots + (n0 + n) % kDSlots;
  const int npairs = gridDim.x * kPairs;
  const int chunks = phase_chunks(p);
  const int t = gp + (n / chunks) * npairs;
  const int j = t / p.tiles_per_expert;
  const int tile = t - j * p.tiles_per_expert;
  const int rowbase = tb.act_e[j] * p.N;
  const int c = n % chunks;
  const uint32_t wbytes = box_lines(p.K) * 1024, abytes = abox_floats(p.K) * 32;
  mbar_arrive_expect_tx(bar, 2 * (wbytes + abytes));
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r0 = rowbase + group_row(p, tile, h);
    tma_load_3d(slot + h * kWBoxCap, p.wmap, 0, r0, c * (kDChunk / 256), bar);
    tma_load_2d(slot + 2 * kWBoxCap + h * kABoxCap, p.amap, c * (kDChunk / 64), r0, bar);
  }
}

// The first kDSlots items of the pair's phase (pair leader only).
__device__ __forceinline__ void issue_head(const Phase& p, const Tables& tb, char* smem, int nact, int gp, int n0) {
  const int total = phase_items(p, nact, gp);
  for (int n = 0; n < kDSlots && n < total; ++n) issue_item(p, tb, smem, gp, n, n0);
}

// Byte offset of lane (row r, quad lane q)'s 8-byte piece of block bc (of the chunk) in a weight
// box whose shared address is 1024-aligned: line bc / 4 holds blocks 4 (bc / 4) .. +3.
__device__ __forceinline__ int wofs(int r, int q, int bc) {
  const int unit = (((bc & 3) << 1) | (q >> 1)) ^ r;
  return (bc >> 2) * 1024 + r * 128 + (unit << 4) + ((q & 1) << 3);
}

// One phase of streamed tiles for this pair; its items run through one slot and one mbarrier
// whose phase parity `n_run` keeps across phases.
template <int NT>
__device__ void stream_phase(const Phase& p, const Tables& tb, int nact, char* smem, int& n_run, bool& dead,
                             int* cta_err, bool head_issued, int trace_slot) {
  char* lut = smem + DSmem::lut;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int pair = warp >> 1, member = warp & 1;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  char* slots = smem + DSmem::slots + pair * kDSlots * kDSlotBytes;
  float* red = reinterpret_cast<float*>(smem + DSmem::red) + pair * 32 * 8;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DSmem::bars) + pair * kDSlots;
  const bool leader = member == 0 && lane == 0;
  const int npairs = gridDim.x * kPairs;
  const int chunks = phase_chunks(p);
  const int gp = blockIdx.x * kPairs + pair;
  const int total_items = phase_items(p, nact, gp);
  const int n0 = n_run;
  const bool swiglu = p.epilogue == E4B_EPI_SWIGLU;
  const int arow = abox_floats(p.K) * 4;  // bytes per absmax box row
  (void)trace_slot;
  if (leader && !dead && !head_issued) issue_head(p, tb, smem, nact, gp, n0);

  int row0 = 0, M = 0, tile = 0;
  float acc[NT][4];
  for (int n = 0; n < total_items; ++n) {
    const int c = n % chunks;
    if (c == 0) {
      const int t = gp + (n / chunks) * npairs;
      const int j = t / p.tiles_per_expert;
      tile = t - j * p.tiles_per_expert;
      row0 = tb.act_row0[j];
      M = tb.act_cnt[j];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] = 0.f;
    }
    const int gn = n0 + n;
    char* slot = slots + (gn % kDSlots) * kDSlotBytes;
    if (!dead && !mbar_wait(&bars[gn % kDSlots], (gn / kDSlots) & 1)) {
      cta_raise(cta_err, E4B_ERR_TIMEOUT);
      dead = true;
    }
    if (n == 0) PTRACE(trace_slot);
    if (!dead) {
      // blocks of this chunk; the members take alternate groups of four (the streaming GEMV's split,
      // so both kernels accumulate in the same order)
      const int nb = min(kDChunk, p.K - c * kDChunk) / 64;
      const __half* xrow[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int m = nt * 8 + gq;
        const int sr = row0 + (m < M ? m : 0);
        const int src = p.x_mapped ? tb.sorted_tok[sr] : sr;
        xrow[nt] = p.x + src * p.xpitch + c * kDChunk + q * 16;
      }
      const char* wA = slot;
      const char* wB = slot + kWBoxCap;
      const char* aA = slot + 2 * kWBoxCap;
      const char* aB = slot + 2 * kWBoxCap + kABoxCap;
      for (int b0 = 4 * member; b0 < nb; b0 += 8) {
        uint2 wa[4], wb[4];
        float sa[4], sb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int b = b0 + i < nb ? b0 + i : b0;
          wa[i] = *reinterpret_cast<const uint2*>(wA + wofs(gq, q, b));
          wb[i] = *reinterpret_cast<const uint2*>(wB + wofs(gq, q, b));
          sa[i] = *reinterpret_cast<const float*>(aA + aofs(gq, b, arow));
          sb[i] = *reinterpret_cast<const float*>(aB + aofs(gq, b, arow));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int b = b0 + i;
          if (b >= nb) break;
          uint4 xf[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            xf[nt][0] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64);
            xf[nt][1] = *reinterpret_cast<const uint4*>(xrow[nt] + b * 64 + 8);
          }
          float pp[NT][4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint32_t w0 = jj < 2 ? wa[i].x : wa[i].y, w1 = jj < 2 ? wb[i].x : wb[i].y;
            uint32_t a0, a1, a2, a3;
            if (jj & 1) {
              a0 = lut2<2>(lut, w0, lane4); a2 = lut2<3>(lut, w0, lane4);
              a1 = lut2<2>(lut, w1, lane4); a3 = lut2<3>(lut, w1, lane4);
            } else {
              a0 = lut2<0>(lut, w0, lane4); a2 = lut2<1>(lut, w0, lane4);
              a1 = lut2<0>(lut, w1, lane4); a3 = lut2<1>(lut, w1, lane4);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xf[nt][jj >> 1]);
              if (jj == 0)
                mma16816_zero(pp[nt], a0, a1, a2, a3, xw[0], xw[1]);
              else
                mma16816(pp[nt], a0, a1, a2, a3, xw[(jj & 1) * 2], xw[(jj & 1) * 2 + 1]);
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            acc[nt][0] = fmaf(pp[nt][0], sa[i], acc[nt][0]);
            acc[nt][1] = fmaf(pp[nt][1], sa[i], acc[nt][1]);
            acc[nt][2] = fmaf(pp[nt][2], sb[i], acc[nt][2]);
            acc[nt][3] = fmaf(pp[nt][3], sb[i], acc[nt][3]);
          }
        }
      }
    }
    const bool last = c == chunks - 1;
    if (last && member == 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) red[(nt * 4 + r) * 32 + lane] = acc[nt][r];
    }
    // both members are done reading the slot; the proxy fence orders those generic reads before
    // the slot's refill by the async proxy
    fence_proxy_async();
    named_barrier(1 + pair, 64);
    if (leader && !dead && n + kDSlots < total_items) issue_item(p, tb, smem, gp, n + kDSlots, n0);
    if (last && member == 0 && !dead) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[nt][r] += red[(nt * 4 + r) * 32 + lane];
      const int rA = group_row(p, tile, 0) + gq, rB = group_row(p, tile, 1) + gq;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m = nt * 8 + 2 * q + h;
          if (m >= M) continue;
          const int srow = row0 + m;
          float va = acc[nt][h], vb = acc[nt][2 + h];
          if (p.x_mapped) {
            const float sc = tb.xscale[tb.sorted_tok[srow]];
            va *= sc;
            vb *= sc;
          }
          __half* o = p.out + (int64_t)srow * p.Nout;
          if (swiglu) {
            o[tile * 8 + gq] = store_cast<__half>(silu_f32(va) * vb, cta_err);
          } else if (p.epilogue == E4B_EPI_SILU) {
            o[rA] = store_cast<__half>(silu_f32(va), cta_err);
            o[rB] = store_cast<__half>(silu_f32(vb), cta_err);
          } else {
            o[rA] = store_cast<__half>(va, cta_err);
            o[rB] = store_cast<__half>(vb, cta_err);
          }
        }
    }
  }
  if (dead && leader)  // drain what may still be in flight, bounded
    for (int m = total_items - kDSlots; m < total_items; ++m)
      if (m >= 0) (void)mbar_wait(&bars[(n0 + m) % kDSlots], ((n0 + m) / kDSlots) & 1);
  if (total_items > 0) PTRACE(trace_slot + 1);
  n_run = n0 + total_items;
}

// The routing tables at DSmem::tables.
__device__ __forceinline__ Tables tables_of(char* smem) {
  Tables tb;
  int* ti = reinterpret_cast<int*>(smem + DSmem::tables);
  tb.pick_e = ti;
  tb.sorted_e = ti + kMaxPicks;
  tb.sorted_tok = ti + 2 * kMaxPicks;
  tb.inv = ti + 3 * kMaxPicks;
  tb.act_e = ti + 4 * kMaxPicks;
  tb.act_row0 = ti + 5 * kMaxPicks;
  tb.act_cnt = ti + 6 * kMaxPicks;
  tb.xscale = reinterpret_cast<float*>(ti + 7 * kMaxPicks);
  tb.misc = ti + 7 * kMaxPicks + 16;
  tb.w = reinterpret_cast<float*>(ti + 7 * kMaxPicks + 32);
  tb.rowmax = reinterpret_cast<unsigned*>(ti + 8 * kMaxPicks + 32);
  return tb;
}

// Phase 0 of both one-launch decode kernels, from kernel entry to the first streamed tile: the
// (fused or given) routing, the stable expert-major permutation of fast.py:126-133 in shared
// memory, the NF4 pair table and the token rows as fp16 with per-row power-of-two scales.
// `issue_first(tb, nact)` runs on every thread right after the permutation is known (the caller's
// copy leaders start their first weight copies there). Returns the number of active experts; the
// CTA is synchronised on return. The caller initialises its mbarriers (thread 0) before the call.
template <class IssueFirst>
__device__ __forceinline__ int decode_prologue(const DecodeArgs& a, char* smem, const Tables& tb,
                                               IssueFirst&& issue_first) {
  namespace cg = cooperative_groups;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = a.T * a.k;
  // the router rows this warp's logit tasks read, into L2 while the token rows load (grid-wide
  // split only: there each warp has at most a few tasks)
  if (a.router_w && a.router_logits && a.cluster <= 1) {
    const int tasks = a.E * ((a.T + kRouterTT - 1) / kRouterTT);
    const int esz = a.router_w_dtype == E4B_F32 ? 4 : 2;
    for (int task = warp * (int)gridDim.x + blockIdx.x; task < tasks; task += kWarps * (int)gridDim.x) {
      const char* row = static_cast<const char*>(a.router_w) + (int64_t)(task % a.E) * a.H * esz;
      for (int off = lane * 128; off < a.H * esz; off += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(row + off));
    }
  }
  // token rows into registers first: their latency overlaps the permutation below
  const int xvec = a.T * (a.H / 8);
  uint4 xr[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int v = tid + i * kThreads;
    if (v < xvec) xr[i] = reinterpret_cast<const uint4*>(a.hidden)[v];
  }
  __half* xs = reinterpret_cast<__half*>(smem + DSmem::x);
  const int xpitch = a.H + 8;

  // ---- phase 0: the permutation first, so the weight stream starts early ------------------
  if (tid == 0) tb.misc[1] = 0;
  if (tid < 16) tb.rowmax[tid] = 0u;
  // the pair table and the token rows as fp16 (with the per-row power-of-two scale of convert.cuh):
  // neither depends on the routing, so with the fused router they fill the wait at its grid barrier
  auto prep = [&]() {
    {  // pair table
      char* lut = smem + DSmem::lut;
      const float code = c_nf4[lane & 15];
#pragma unroll 4
      for (int e = warp; e < 256; e += kWarps) {
        const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
        reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
      }
    }
    DTRACE(11);
    {  // token rows -> fp16 with the per-row power-of-two scale of convert.cuh
      float v[2][8];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int vi = tid + i * kThreads;
        // a warp's 32 vectors lie in one row (H / 8 is a multiple of 32): reduce, then one atomic
        if (i * kThreads + warp * 32 < xvec) {
          float m = 0.f;
          if (vi < xvec) {
            unpack8(xr[i], a.act_dtype, v[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
          }
#pragma unroll
          for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) atomicMax(&tb.rowmax[vi / (a.H / 8)], __float_as_uint(m));
        }
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int vi = tid + i * kThreads;
        if (vi < xvec) {
          const int r = vi / (a.H / 8), c8 = vi - r * (a.H / 8);
          const float m = __uint_as_float(tb.rowmax[r]);
          int sh = 0;
          if (m > 32768.f) {
            int ex;
            frexpf(m / 32768.f, &ex);
            sh = ex;
          }
          const float inv = ldexpf(1.f, -sh);
          uint4 o;
          uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int j = 0; j < 4; ++j) ow[j] = pack2<__half>(v[i][2 * j] * inv, v[i][2 * j + 1] * inv);
          *reinterpret_cast<uint4*>(xs + r * xpitch + c8 * 8) = o;
          if (c8 == 0) tb.xscale[r] = ldexpf(1.f, sh);
        }
      }
    }
  };
  if (a.router_w) {
    // ---- fused router: logits into shared memory (spread over the grid through global
    // scratch and a grid barrier, or computed by every CTA), then the same top-k everywhere ----
    float* logits = reinterpret_cast<float*>(smem + DSmem::logits);
    const int ttiles = (a.T + kRouterTT - 1) / kRouterTT, tasks = a.E * ttiles;
    const bool w16 = a.router_w_dtype != E4B_F32;  // 16-bit weights: all strips of a lane in flight
    // In clusters the (expert, token tile) tasks are split over the cluster's CTAs; with global
    // scratch they are spread one warp per SM across the grid and shared through a grid barrier;
    // otherwise every CTA computes all of them.
    // the token rows (raw, already in registers) into the not yet used copy slots: the logit tasks
    // read them from shared memory instead of every warp of the grid hitting the same lines of L2
    uint16_t* xraw = reinterpret_cast<uint16_t*>(smem + DSmem::slots);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int v = tid + i * kThreads;
      if (v < xvec) reinterpret_cast<uint4*>(xraw)[v] = xr[i];
    }
    __syncthreads();
    const bool in_cluster = a.cluster > 1;
    const int crank = in_cluster ? (int)cg::this_cluster().block_rank() : 0;
    float* dst = (a.router_logits && !in_cluster) ? a.router_logits : logits;
    const int w0 = in_cluster ? crank + a.cluster * warp : a.router_logits ? warp * (int)gridDim.x + blockIdx.x : warp;
    const int wstep = in_cluster ? a.cluster * kWarps : a.router_logits ? kWarps * (int)gridDim.x : kWarps;
    for (int task = w0; task < tasks; task += wstep) {
      if (w16)
        router_logits_warp16<8>(xraw, a.act_dtype, a.router_w, a.router_w_dtype, a.T, a.H, a.E, task % a.E,
                                (task / a.E) * kRouterTT, dst);
      else
        router_logits_warp(xraw, a.act_dtype, a.router_w, a.router_w_dtype, a.T, a.H, a.E, task % a.E,
                           (task / a.E) * kRouterTT, dst);
    }
    __syncthreads();  // rowmax cleared
    prep();
    if (in_cluster) {
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();
      for (int i = tid; i < a.T * a.E; i += kThreads) {  // the peers' logits into this CTA's copy
        const int owner = (((i / a.E) / kRouterTT) * a.E + i % a.E) % a.cluster;
        if (owner != crank) logits[i] = *cl.map_shared_rank(logits + i, owner);
      }
      // peers keep their logits until every CTA of the cluster has read them: the matching wait
      // is the kernel's last statement
      asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    } else if (a.router_logits) {
      cg::this_grid().sync();
      for (int i = tid; i < a.T * a.E; i += kThreads) logits[i] = __ldcg(a.router_logits + i);
    }
    DTRACE(14);
    __syncthreads();
    DTRACE(15);
    if (warp < a.T) {
      int se = 0;
      float sw = 0.f;
      // selection slots per token warp in the (not yet used) reduction area: 32 values + 32 ids
      float* sv = reinterpret_cast<float*>(smem + DSmem::red) + warp * 64;
      int* si = reinterpret_cast<int*>(sv + 32);
#define E4B_DTOPK(EPL) \
  router_topk_warp_ranked<EPL>(logits, a.T, a.E, a.k, a.route_kind, a.renorm, warp, sv, si, se, sw)
      if (a.E <= 32) E4B_DTOPK(1);
      else if (a.E <= 64) E4B_DTOPK(2);
      else if (a.E <= 128) E4B_DTOPK(4);
      else if (a.E <= 256) E4B_DTOPK(8);
      else E4B_DTOPK(32);
#undef E4B_DTOPK
      if (lane < a.k) {
        tb.pick_e[warp * a.k + lane] = se;
        tb.w[warp * a.k + lane] = sw;
        if (blockIdx.x == 0) {
          a.topk_idx_out[warp * a.k + lane] = se;
          a.topk_w_out[warp * a.k + lane] = sw;
        }
      }
    }
    DTRACE(16);
  } else if (tid < R) {
    int* errw = &tb.misc[1];
    tb.pick_e[tid] = stack_expert(a.topk_idx[tid], a.emap, a.routed, a.E, blockIdx.x == 0 ? errw : nullptr,
                                  blockIdx.x == 0);
    tb.w[tid] = load_as_f32(a.topk_w, a.w_dtype, tid);
  }
  __syncthreads();
  DTRACE(17);
  if (tid < R) {  // stable rank by (expert, flat index): the permutation of fast.py:126-133
    const int e = tb.pick_e[tid];
    int rank = 0;
    for (int j = 0; j < R; ++j) {
      const int ej = tb.pick_e[j];
      rank += (ej < e) | ((ej == e) & (j < tid));
    }
    tb.sorted_e[rank] = e;
    tb.sorted_tok[rank] = tid / a.k;
    tb.inv[tid] = rank;
  }
  __syncthreads();
  DTRACE(18);
  bool start = false;
  unsigned ball = 0;
  if (warp < kMaxPicks / 32) {
    start = tid < R && (tid == 0 || tb.sorted_e[tid - 1] != tb.sorted_e[tid]);
    ball = __ballot_sync(0xffffffffu, start);
    if (lane == 0) tb.misc[2 + warp] = __popc(ball);
  }
  __syncthreads();
  if (warp < kMaxPicks / 32) {
    int before = 0;
    for (int w = 0; w < warp; ++w) before += tb.misc[2 + w];
    const int idx = before + __popc(ball & ((1u << lane) - 1u));
    if (start) {
      tb.act_e[idx] = tb.sorted_e[tid];
      tb.act_row0[idx] = tid;
    }
    if (tid == 0) tb.misc[0] = tb.misc[2] + tb.misc[3] + tb.misc[4] + tb.misc[5];
  }
  __syncthreads();
  const int nact = tb.misc[0];
  DTRACE(1);
  issue_first(tb, nact);
  if (tid < nact) tb.act_cnt[tid] = (tid + 1 < nact ? tb.act_row0[tid + 1] : R) - tb.act_row0[tid];
  DTRACE(10);
  if (!a.router_w) prep();
  DTRACE(12);
  __syncthreads();
  DTRACE(13);
  return nact;
}

template <typename OutT, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_decode_layer_kernel(DecodeArgs a, const __grid_constant__ CUtensorMap wmap_gu,
                            const __grid_constant__ CUtensorMap amap_gu, const __grid_constant__ CUtensorMap wmap_dn,
                            const __grid_constant__ CUtensorMap amap_dn) {
  extern __shared__ __align__(1024) char smem[];
  namespace cg = cooperative_groups;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int R = a.T * a.k;
  DTRACE(0);
  if (tid < 4) {  // descriptors into the TMA unit's cache before the first copies
    const CUtensorMap* m = tid == 0 ? &wmap_gu : tid == 1 ? &amap_gu : tid == 2 ? &wmap_dn : &amap_dn;
    asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
  }
  const Tables tb = tables_of(smem);
  int* cta_err = &tb.misc[1];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + DSmem::bars);
  __half* xs = reinterpret_cast<__half*>(smem + DSmem::x);
  const int xpitch = a.H + 8;

  Phase pa{};
  pa.wmap = &wmap_gu;
  pa.amap = &amap_gu;
  pa.N = a.has_gate ? 2 * a.I : a.I;
  pa.K = a.H;
  pa.epilogue = a.has_gate ? E4B_EPI_SWIGLU : E4B_EPI_SILU;
  pa.tiles_per_expert = pa.N / 16;
  pa.x = xs;
  pa.xpitch = xpitch;
  pa.x_mapped = true;
  pa.out = a.h;
  pa.Nout = a.I;

  if (tid == 0) {
    for (int s = 0; s < kPairs * kDSlots; ++s) mbar_init(&bars[s], 1);
    fence_proxy_async();
  }
  const int nact = decode_prologue(a, smem, tb, [&](const Tables& t, int na) {
    if ((warp & 1) == 0 && lane == 0)  // pair leaders: the first gate_up items
      issue_head(pa, t, smem, na, blockIdx.x * kPairs + (warp >> 1), 0);
  });

  // ---- phase A: gate_up --------------------------------------------------------------------
  int n_run = 0;
  bool dead = false;
  DTRACE(2);
  stream_phase<NT>(pa, tb, nact, smem, n_run, dead, cta_err, true, 0);
  // phase B's weights do not depend on phase A: each pair starts its first down item now, so the
  // copy overlaps the grid barrier
  Phase pb{};
  pb.wmap = &wmap_dn;
  pb.amap = &amap_dn;
  pb.N = a.H;
  pb.K = a.I;
  pb.epilogue = E4B_EPI_NONE;
  pb.tiles_per_expert = a.H / 16;
  pb.x = a.h;
  pb.xpitch = a.I;
  pb.x_mapped = false;
  pb.out = a.down_rows;
  pb.Nout = a.H;
  if ((warp & 1) == 0 && lane == 0 && !dead) issue_head(pb, tb, smem, nact, blockIdx.x * kPairs + (warp >> 1), n_run);
  DTRACE(3);
  cg::this_grid().sync();
  DTRACE(4);

  // ---- phase B: down -----------------------------------------------------------------------
  if ((int64_t)R * (a.I + 8) * 2 <= kDXBudget) {  // all of h fits where the token rows were: stage it
    const int hp = a.I + 8, vec = a.I / 8;
    for (int v = tid; v < R * vec; v += kThreads) {
      const int r = v / vec, c = v - r * vec;
      *reinterpret_cast<uint4*>(xs + r * hp + c * 8) = *reinterpret_cast<const uint4*>(a.h + (int64_t)r * a.I + c * 8);
    }
    __syncthreads();
    pb.x = xs;
    pb.xpitch = hp;
  }
  DTRACE(5);
  stream_phase<NT>(pb, tb, nact, smem, n_run, dead, cta_err, true, 2);
  DTRACE(6);
  __syncthreads();
  if (tid == 0) a.cta_err[blockIdx.x] = tb.misc[1];
  cg::this_grid().sync();
  DTRACE(7);

  // errors of phases 0-B: the first failing CTA's code (CTA 0, parallel reads)
  auto fold_errors = [&]() {
    if (blockIdx.x != 0) return;
    if (tid == 0) tb.misc[7] = 0x7fffffff;
    __syncthreads();
    for (int b = tid; b < (int)gridDim.x; b += kThreads)
      if (a.cta_err[b]) atomicMin(&tb.misc[7], b);
    __syncthreads();
    if (tid == 0 && tb.misc[7] != 0x7fffffff) atomicCAS(a.err, 0, a.cta_err[tb.misc[7]]);  // sticky word
  };
  fold_errors();

  // ---- phase C: out[t] = sum over slots, in order, of fp32(down[inv[t*k+s]]) * w[t,s] ----------
  const int vecs = a.T * (a.H / 8);
  for (int v = blockIdx.x * kThreads + tid; v < vecs; v += gridDim.x * kThreads) {
    const int t = v / (a.H / 8), h8 = (v - t * (a.H / 8)) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int s0 = 0; s0 < a.k; s0 += 8) {
      uint4 d[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < a.k)
          d[u] = *reinterpret_cast<const uint4*>(a.down_rows + (int64_t)tb.inv[t * a.k + s0 + u] * a.H + h8);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + u >= a.k) break;
        const __half* dv = reinterpret_cast<const __half*>(&d[u]);
        const float ws = tb.w[t * a.k + s0 + u];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(__half2float(dv[i]), ws, acc[i]);  // slot order
      }
    }
    OutT* o = reinterpret_cast<OutT*>(a.out) + (int64_t)t * a.H + h8;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = store_cast_out<OutT>(acc[i], cta_err);
  }
  DTRACE(8);
  if (a.out_dtype == E4B_F16) {  // fp16 outputs can saturate in phase C: fold once more
    __syncthreads();
    if (tid == 0) a.cta_err[blockIdx.x] = tb.misc[1];
    cg::this_grid().sync();
    fold_errors();
  }
  DTRACE(9);
}

// ---- slice kernel -----------------------------------------------------------------------------
// The layer for 1..8 tokens as independent units of one active expert x 64 intermediate columns
// (one absmax block of a down row): a CTA streams the unit's 64 gate + 64 up rows over all of H,
// reduces them across its warps into the unit's 64 h values (SwiGLU, fp16), then streams the
// unit's 64-column strip of every down row and stores fp32 partial down rows per (pick, strip).
// No unit waits on another CTA, so gate_up and down run back to back without a grid barrier; one
// grid barrier before the combine, which sums the strips of each pick in strip order, rounds the
// sum to fp16 (the down_rows rounding of the multi-kernel path) and weights the picks in slot order.
//
// Copies run through a ring of kSSlots stages filled by thread 0: a gate_up stage is 512 K
// elements of the unit's 128 rows (two 16 KB boxes of [2 lines][64 rows][128 B], 128-byte
// swizzle, and two [64 rows][8 floats] absmax boxes), a down stage 512 rows of the strip (two
// [256 rows][32 B] boxes and two [256 rows][4 floats] absmax boxes, the strip's float among the
// four). In a gate_up stage warp w owns block w / 2 of the stage for tiles 4 (w % 2) .. +3 (a tile
// is 8 gate rows and the 8 matching up rows), so its token fragments are read once per stage; in
// a down stage it owns tiles 2w, 2w + 1 (16 rows each) with the unit's h fragment in registers.
// The per-block arithmetic (pair-table decode, mma.sync m16n8k16, fp32 absmax scaling) is the
// streaming GEMV's; the blocks of a gate_up row are summed per warp and then across warps in warp
// order, so the result is deterministic but not bit-identical to the phase kernel's.
constexpr int kSW = 64;          // intermediate columns per unit
constexpr int kSGK = 512;        // K elements per gate_up stage
constexpr int kSDRows = 512;     // down rows per stage
constexpr int kSSlots = 3;
constexpr int kSSlot = 36 * 1024;
constexpr int kSHPitch = kSW + 8;  // halves per h row in shared memory

struct SSmem {
  static constexpr int ring = DSmem::slots;                 // 1024-aligned
  static constexpr int red = ring + kSSlots * kSSlot;       // [warp][16][32] fp32 partial tiles
  static constexpr int hs = red + kWarps * 16 * 32 * 4;     // [8 tokens][kSHPitch] fp16
  static constexpr int end = hs + 8 * kSHPitch * 2;
};
// the combine stages [R][ceil(H / 4 / grid)][I / 64] float4 strips in the ring (R <= 64 here)
static_assert(SSmem::ring % 1024 == 0 && kSSlot % 1024 == 0, "swizzled boxes need 1024-byte alignment");
static_assert(SSmem::end <= DSmem::bars, "slice layout overlaps the barriers");
static_assert(2 * kSSlots * 8 + kSSlots * 4 <= kPairs * kDSlots * 8, "slice barriers and release counters fit");

__device__ __forceinline__ void slice_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

struct SliceMaps {
  const CUtensorMap* gw;  // gate_up packed [lines][rows][128 B], box {128, 64, 2}
  const CUtensorMap* ga;  // gate_up absmax [rows][H / 64], box {8, 64}, 32-byte swizzle
  const CUtensorMap* dw;  // down packed [rows][I / 2], box {32, 256}
  const CUtensorMap* da;  // down absmax [rows][I / 64], box {4, 256}
};

// Copies of this CTA's stage n into ring slot n % kSSlots (thread 0 only).
__device__ __forceinline__ void slice_issue(const DecodeArgs& a, const SliceMaps& m, const Tables& tb, char* smem,
                                            int n, int nsl, int ng, int spu) {
  const int ui = n / spu, st = n - ui * spu;
  const int u = blockIdx.x + ui * (int)gridDim.x;
  const int j = u / nsl, s = u - j * nsl;
  const int e = tb.act_e[j];
  char* slot = smem + SSmem::ring + (n % kSSlots) * kSSlot;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DSmem::bars) + (n % kSSlots);
  if (st < ng) {
    const int r0 = e * 2 * a.I + s * kSW, r1 = r0 + a.I;
    mbar_arrive_expect_tx(full, 2 * 16384 + 2 * 2048);
    tma_load_3d(slot, m.gw, 0, r0, 2 * st, full);
    tma_load_3d(slot + 16384, m.gw, 0, r1, 2 * st, full);
    tma_load_2d(slot + 32768, m.ga, 8 * st, r0, full);
    tma_load_2d(slot + 34816, m.ga, 8 * st, r1, full);
  } else {
    const int r0 = e * a.H + (st - ng) * kSDRows;
    mbar_arrive_expect_tx(full, 16384 + 8192);
    tma_load_2d(slot, m.dw, 32 * s, r0, full);
    tma_load_2d(slot + 8192, m.dw, 32 * s, r0 + 256, full);
    tma_load_2d(slot + 16384, m.da, 4 * (s >> 2), r0, full);
    tma_load_2d(slot + 20480, m.da, 4 * (s >> 2), r0 + 256, full);
  }
}

// One 64-element block of a 16-row tile against one token fragment: rows A (w0, scale sa) and
// B (w1, scale sb), the streaming GEMV's fragment order. PW of the block's first-half words
// (w0v.x, then w1v.x) are decoded in registers, the rest through the shared pair table: the
// split balances the shared-memory pipe against the integer pipe.
template <int PW>
__device__ __forceinline__ void slice_block(float (&acc)[4], const char* lut, uint2 w0v, uint2 w1v, float sa,
                                            float sb, const uint4 (&xf)[2], uint32_t lane4, const Nf4Bytes& T) {
  uint32_t r0[4], r1[4];  // register-decoded pairs of w0v.x / w1v.x (entries 0..3 = bytes 0..3)
  if (PW >= 1) nf4_decode_word(w0v.x, T, r0);
  if (PW >= 2) nf4_decode_word(w1v.x, T, r1);
  float pp[4];
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const uint32_t w0 = jj < 2 ? w0v.x : w0v.y, w1 = jj < 2 ? w1v.x : w1v.y;
    uint32_t a0, a1, a2, a3;
    if (jj & 1) {
      a0 = (jj < 2 && PW >= 1) ? r0[2] : lut2<2>(lut, w0, lane4);
      a2 = (jj < 2 && PW >= 1) ? r0[3] : lut2<3>(lut, w0, lane4);
      a1 = (jj < 2 && PW >= 2) ? r1[2] : lut2<2>(lut, w1, lane4);
      a3 = (jj < 2 && PW >= 2) ? r1[3] : lut2<3>(lut, w1, lane4);
    } else {
      a0 = (jj < 2 && PW >= 1) ? r0[0] : lut2<0>(lut, w0, lane4);
      a2 = (jj < 2 && PW >= 1) ? r0[1] : lut2<1>(lut, w0, lane4);
      a1 = (jj < 2 && PW >= 2) ? r1[0] : lut2<0>(lut, w1, lane4);
      a3 = (jj < 2 && PW >= 2) ? r1[1] : lut2<1>(lut, w1, lane4);
    }
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xf[jj >> 1]);
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

template <typename OutT, int PW>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_decode_slice_kernel(DecodeArgs a, const __grid_constant__ CUtensorMap gw, const __grid_constant__ CUtensorMap ga,
                            const __grid_constant__ CUtensorMap dw, const __grid_constant__ CUtensorMap da) {
  extern __shared__ __align__(1024) char smem[];
  namespace cg = cooperative_groups;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, q = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  DTRACE(0);
  if (tid < 4) {
    const CUtensorMap* mp = tid == 0 ? &gw : tid == 1 ? &ga : tid == 2 ? &dw : &da;
    asm volatile("prefetch.tensormap [%0];" ::"l"(mp) : "memory");
  }
  const Tables tb = tables_of(smem);
  int* cta_err = &tb.misc[1];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + DSmem::bars);
  uint64_t* empty = full + kSSlots;
  int* relcnt = reinterpret_cast<int*>(empty + kSSlots);  // [kSSlots] warps done with each slot
  const char* lut = smem + DSmem::lut;
  const __half* xs = reinterpret_cast<const __half*>(smem + DSmem::x);
  const int xpitch = a.H + 8;
  float* red = reinterpret_cast<float*>(smem + SSmem::red);
  __half* hs = reinterpret_cast<__half*>(smem + SSmem::hs);
  const SliceMaps maps{&gw, &ga, &dw, &da};
  const Nf4Bytes nfb = nf4_bytes();
  const int nsl = a.I / kSW, ng = a.H / kSGK, nd = a.H / kSDRows, spu = ng + nd;
  if (tid == 0) {
    for (int s = 0; s < kSSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
      relcnt[s] = 0;
    }
    fence_proxy_async();
  }
  int total = 0;  // this CTA's stages
  const int nact = decode_prologue(a, smem, tb, [&](const Tables& t, int na) {
    const int units = na * nsl;
    const int mine = units > (int)blockIdx.x ? (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    if (tid == 0)
      for (int n = 0; n < kSSlots && n < mine * spu; ++n) slice_issue(a, maps, t, smem, n, nsl, ng, spu);
  });
  {
    const int units = nact * nsl;
    const int mine = units > (int)blockIdx.x ? (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    total = mine * spu;
  }
  DTRACE(2);
  bool dead = false;
  int n = 0;
  for (int ui = 0; n < total; ++ui) {
    const int u = blockIdx.x + ui * (int)gridDim.x;
    const int j = u / nsl, s = u - j * nsl;
    const int row0 = tb.act_row0[j], M = tb.act_cnt[j];
    auto wait_full = [&](int nn) {
      if (!dead && !mbar_wait(&full[nn % kSSlots], (nn / kSSlots) & 1)) {
        cta_raise(cta_err, E4B_ERR_TIMEOUT);
        dead = true;
      }
      if (nn < 8) {
        STRACE(1, nn);
        STRACE(15, 24 + nn);
      }
    };
    auto release = [&](int nn) {
      if (!(a.slice_flags & 1)) fence_proxy_async();
      __syncwarp();
      if (a.slice_flags & 2) {
        // the last of the 16 warps to finish with the slot refills it: no warp waits for the others
        if (lane == 0) {
          __threadfence_block();
          if (atomicAdd(&relcnt[nn % kSSlots], 1) == kWarps - 1) {
            relcnt[nn % kSSlots] = 0;
            __threadfence_block();
            if (nn + kSSlots < total && !dead) {
              fence_proxy_async();  // the other warps' reads of the slot before the async-proxy refill
              slice_issue(a, maps, tb, smem, nn + kSSlots, nsl, ng, spu);
            }
          }
        }
        if (nn < 8) STRACE(1, 8 + nn);
        return;
      }
      if (lane == 0) slice_arrive(&empty[nn % kSSlots]);
      if (nn < 8) STRACE(1, 8 + nn);
      if (tid == 0 && nn + kSSlots < total && !dead) {
        if (mbar_wait(&empty[nn % kSSlots], (nn / kSSlots) & 1))
          slice_issue(a, maps, tb, smem, nn + kSSlots, nsl, ng, spu);
        else
          cta_raise(cta_err, E4B_ERR_TIMEOUT);  // the consumers time out on the missing stages
        if (nn < 8) STRACE(0, 16 + nn);
      }
    };
    // ---- gate_up: 128 rows x H ----
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][c] = 0.f;
    const int bl = warp >> 1, tset = (warp & 1) * 4;
    const int src = tb.sorted_tok[row0 + (gq < M ? gq : 0)];
    for (int st = 0; st < ng; ++st, ++n) {
      wait_full(n);
      if (n == 0) DTRACE(6);
      if (!dead) {
        const char* slot = smem + SSmem::ring + (n % kSSlots) * kSSlot;
        uint4 xf[2];
        const __half* xrow = xs + src * xpitch + st * kSGK + bl * 64 + q * 16;
        xf[0] = *reinterpret_cast<const uint4*>(xrow);
        xf[1] = *reinterpret_cast<const uint4*>(xrow + 8);
        uint2 wa[4], wb[4];
        float sa[4], sb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = (tset + i) * 8 + gq;
          const int unit = (((bl & 3) << 1) | (q >> 1)) ^ (rr & 7);
          const int wo = (bl >> 2) * 8192 + rr * 128 + (unit << 4) + ((q & 1) << 3);
          wa[i] = *reinterpret_cast<const uint2*>(slot + wo);
          wb[i] = *reinterpret_cast<const uint2*>(slot + 16384 + wo);
          sa[i] = *reinterpret_cast<const float*>(slot + 32768 + aofs(rr, bl, 32));
          sb[i] = *reinterpret_cast<const float*>(slot + 34816 + aofs(rr, bl, 32));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) slice_block<PW>(acc[i], lut, wa[i], wb[i], sa[i], sb[i], xf, lane4, nfb);
      }
      release(n);
    }
    // ---- reduce across the 8 warps of each tile; h = silu(gate) * up for the unit's tokens ----
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) red[(warp * 16 + i * 4 + c) * 32 + lane] = acc[i][c];
    __syncthreads();
    {
      const int t = tid >> 6, hh = (tid >> 5) & 1, i = t & 3;
      float g = 0.f, up = 0.f;
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const int w = (t >> 2) + 2 * v;
        g += red[(w * 16 + i * 4 + hh) * 32 + lane];
        up += red[(w * 16 + i * 4 + 2 + hh) * 32 + lane];
      }
      const int m = 2 * q + hh;
      if (m < M) {
        const float sc = tb.xscale[tb.sorted_tok[row0 + m]];
        hs[m * kSHPitch + t * 8 + gq] = store_cast<__half>(silu_f32(g * sc) * (up * sc), cta_err);
      }
    }
    __syncthreads();
    uint4 hf[2];
    {
      const __half* hrow = hs + (gq < M ? gq : 0) * kSHPitch + q * 16;
      hf[0] = *reinterpret_cast<const uint4*>(hrow);
      hf[1] = *reinterpret_cast<const uint4*>(hrow + 8);
    }
    if (ui == 0) DTRACE(5);
    // ---- down: the unit's strip of all H rows, fp32 partial rows ----
    for (int st = 0; st < nd; ++st, ++n) {
      wait_full(n);
      if (!dead) {
        const char* slot = smem + SSmem::ring + (n % kSSlots) * kSSlot;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int t = 2 * warp + i;
          const int ra = t * 16 + gq, rb = ra + 8;
          const uint2 wa = *reinterpret_cast<const uint2*>(slot + ra * 32 + q * 8);
          const uint2 wb = *reinterpret_cast<const uint2*>(slot + rb * 32 + q * 8);
          const float sa = *reinterpret_cast<const float*>(slot + 16384 + ra * 16 + (s & 3) * 4);
          const float sb = *reinterpret_cast<const float*>(slot + 16384 + rb * 16 + (s & 3) * 4);
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          slice_block<PW>(d, lut, wa, wb, sa, sb, hf, lane4, nfb);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int m = 2 * q + hh;
            if (m < M) {
              float* prow = a.part + ((int64_t)(row0 + m) * nsl + s) * a.H + st * kSDRows;
              prow[ra] = d[hh];
              prow[rb] = d[2 + hh];
            }
          }
        }
      }
      release(n);
    }
  }
  if (tid == 0 && total > 0)  // copies still in flight after a timeout: bounded waits for the last ones
    for (int m = total - kSSlots; m < total; ++m)
      if (m >= 0) (void)mbar_wait(&full[m % kSSlots], (m / kSSlots) & 1);
  (void)dead;
  DTRACE(3);
  __syncthreads();
  if (tid == 0) a.cta_err[blockIdx.x] = tb.misc[1];
  cg::this_grid().sync();
  DTRACE(4);
  auto fold_errors = [&]() {
    if (blockIdx.x != 0) return;
    if (tid == 0) tb.misc[7] = 0x7fffffff;
    __syncthreads();
    for (int b = tid; b < (int)gridDim.x; b += kThreads)
      if (a.cta_err[b]) atomicMin(&tb.misc[7], b);
    __syncthreads();
    if (tid == 0 && tb.misc[7] != 0x7fffffff) atomicCAS(a.err, 0, a.cta_err[tb.misc[7]]);  // sticky word
  };
  fold_errors();
  const bool clean = tb.misc[1] == 0;  // errors before the combine were folded above

  // ---- combine: down row of pick i = fp16(sum over strips, in order); out[t] = sum over slots ----
  const int R = a.T * a.k, H4 = a.H / 4;
  const int per = (H4 + (int)gridDim.x - 1) / (int)gridDim.x;
  const int c0 = blockIdx.x * per, nc = min(per, H4 - c0);
  if (nc > 0) {
    // one float4 load per (pick, column, strip) thread, all in flight at once; then the strips of
    // each (pick, column) summed in strip order from shared memory
    float4* sp = reinterpret_cast<float4*>(smem + SSmem::ring);  // [R][nc][nsl]
    float4* sd = reinterpret_cast<float4*>(smem + SSmem::red);   // [R][nc]
    const int per_pick = nc * nsl;
    for (int v = tid; v < R * per_pick; v += kThreads) {
      const int i = v / per_pick, rem = v - i * per_pick, c = rem / nsl, s = rem - c * nsl;
      sp[v] = __ldcg(reinterpret_cast<const float4*>(a.part + ((int64_t)tb.inv[i] * nsl + s) * a.H) + c0 + c);
    }
    __syncthreads();
    for (int v = tid; v < R * nc; v += kThreads) {
      const float4* p = sp + v * nsl;
      float4 acc4 = p[0];
      for (int s = 1; s < nsl; ++s) {
        const float4 x4 = p[s];
        acc4.x += x4.x;
        acc4.y += x4.y;
        acc4.z += x4.z;
        acc4.w += x4.w;
      }
      acc4.x = __half2float(store_cast<__half>(acc4.x, cta_err));
      acc4.y = __half2float(store_cast<__half>(acc4.y, cta_err));
      acc4.z = __half2float(store_cast<__half>(acc4.z, cta_err));
      acc4.w = __half2float(store_cast<__half>(acc4.w, cta_err));
      sd[v] = acc4;
    }
    __syncthreads();
    for (int v = tid; v < a.T * nc; v += kThreads) {
      const int t = v / nc, c = v - t * nc;
      float o[4] = {0.f, 0.f, 0.f, 0.f};
      for (int sl = 0; sl < a.k; ++sl) {  // slot order
        const float4 d4 = sd[(t * a.k + sl) * nc + c];
        const float ws = tb.w[t * a.k + sl];
        o[0] = fmaf(d4.x, ws, o[0]);
        o[1] = fmaf(d4.y, ws, o[1]);
        o[2] = fmaf(d4.z, ws, o[2]);
        o[3] = fmaf(d4.w, ws, o[3]);
      }
      OutT* op = reinterpret_cast<OutT*>(a.out) + (int64_t)t * a.H + (c0 + c) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) op[i] = store_cast_out<OutT>(o[i], cta_err);
    }
  }
  DTRACE(8);
  // saturation in the combine (fp16 down rows or outputs): into the sticky word directly
  __syncthreads();
  if (tid == 0 && clean && tb.misc[1]) atomicCAS(a.err, 0, tb.misc[1]);
  if (a.cluster > 1 && a.router_w) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

}  // namespace

// One-launch decode kernels: 0 off (multi-kernel path), 1 the flow kernel where it applies and the
// phase kernel elsewhere, 2 the phase kernel only, 3 (the default) the slice kernel where it
// applies and the phase kernel elsewhere. -1: not yet read from E4B_DECODE_KERNEL.
std::atomic<int> g_decode_mode{-1};

int decode_mode() {
  int m = g_decode_mode.load(std::memory_order_relaxed);
  if (m < 0) {
    const char* v = getenv("E4B_DECODE_KERNEL");
    const int env = v ? (v[0] == '0' ? 0 : v[0] == '1' ? 1 : v[0] == '2' ? 2 : 3) : 3;
    int expected = -1;
    g_decode_mode.compare_exchange_strong(expected, env);
    m = g_decode_mode.load(std::memory_order_relaxed);
  }
  return m;
}

size_t decode_layer_sync_bytes(int grid) { return (size_t)grid * sizeof(int); }

static std::mutex g_dl_mu;  // guards the per-device caches below

static int sm_count_cached() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(g_dl_mu);
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev];
}

int decode_layer_grid() { return sm_count_cached(); }

bool decode_router_fusable(const e4b_moe_desc& d) { return (int64_t)d.tokens * d.num_experts <= kMaxLogits; }

bool decode_layer_eligible(const e4b_moe_desc& d) {
  if (decode_mode() == 0) return false;
  if (d.weight_format != E4B_FMT_NF4 || d.lora_rank != 0) return false;
  if (d.tokens < 1 || d.tokens > 16 || (int64_t)d.tokens * d.top_k > kMaxPicks) return false;
  if (d.hidden % 256 || d.intermediate % 256) return false;
  // the absmax boxes are 4, 8, 16 or 32 blocks wide (a power of two under the box swizzle): each
  // K is 256, 512, 1024 or a multiple of 2048
  for (int K : {d.hidden, d.intermediate})
    if (K > 1024 ? K % 2048 : (K & (K - 1))) return false;
  if ((int64_t)d.tokens * (d.hidden + 8) * 2 > kDXBudget) return false;
  if ((int64_t)d.tokens * d.hidden > 2 * kThreads * 8) return false;  // two 16-byte vectors of rows per thread
  if (d.tokens > 16) return false;
  if ((int64_t)d.num_experts * (d.has_gate ? 2 * d.intermediate : d.intermediate) >= (1ll << 31)) return false;
  if ((int64_t)d.num_experts * d.hidden >= (1ll << 31)) return false;
  if (!is_act_dtype(d.act_dtype)) return false;
  return encode_tiled_fn() != nullptr && decode_layer_grid() > 0;
}

static std::atomic<int> g_slice_no_cluster[64];
static void slice_cluster_off(int dev) { g_slice_no_cluster[dev].store(1); }

bool decode_slice_shape(const e4b_moe_desc& d) {
  if (!(d.weight_format == E4B_FMT_NF4 && d.lora_rank == 0 && d.has_gate && d.tokens >= 1 && d.tokens <= 8 &&
        d.hidden % kSGK == 0 && d.intermediate % 256 == 0 && decode_layer_eligible(d)))
    return false;
  // the combine stages each CTA's [R][columns][strips] float4 partials in the copy ring
  const int grid = decode_layer_grid() * 19 / 20;  // the smallest grid a clustered launch takes
  if (grid < 1) return false;
  const int64_t cols = (d.hidden / 4 + grid - 1) / grid;
  return (int64_t)d.tokens * d.top_k * cols * (d.intermediate / kSW) * 16 <= (int64_t)kSSlots * kSSlot;
}

size_t decode_slice_part_bytes(const e4b_moe_desc& d) {
  return (size_t)d.tokens * d.top_k * (d.intermediate / kSW) * d.hidden * 4;
}

template <typename OutT, int NT>
static e4b_status launch_decode(const DecodeArgs& a, cudaStream_t s) {
  static unsigned long long configured = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return E4B_ERR_CUDA;
  const unsigned long long bit = 1ull << dev;
  auto kern = nf4_decode_layer_kernel<OutT, NT>;
  {
    std::lock_guard<std::mutex> lk(g_dl_mu);  // released before decode_layer_grid() takes it again
    if (!(configured & bit)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DSmem::total) != cudaSuccess)
        return E4B_ERR_CUDA;
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, DSmem::total) != cudaSuccess ||
          per_sm < 1)
        return E4B_ERR_UNSUPPORTED;
      configured |= bit;
    }
  }
  const int n1 = a.has_gate ? 2 * a.I : a.I;
  CUtensorMap wgu, agu, wdn, adn;
  auto maps = [&](CUtensorMap& w, CUtensorMap& am, const uint8_t* packed, const float* absmax, int rows_per_e,
                  int K) {
    const cuuint64_t rows = (cuuint64_t)a.E * rows_per_e;
    // packed bytes as [lines (K/256)][rows][128 B]: a box of 8 rows x up to 8 lines lands row-major
    // per line, so the 128-byte swizzle XORs row r's units with r (conflict-free fragment reads)
    const cuuint64_t wdims[3] = {128, rows, (cuuint64_t)(K / 256)};
    const cuuint64_t wstr[2] = {(cuuint64_t)(K / 2), 128};
    const cuuint32_t wbox[3] = {128, 8, (cuuint32_t)box_lines(K)};
    const cuuint64_t adims[2] = {(cuuint64_t)(K / 64), rows};
    const cuuint64_t astr[1] = {(cuuint64_t)(K / 64) * 4};
    const cuuint32_t abox[2] = {(cuuint32_t)abox_floats(K), 8};
    const int S = abox_floats(K) * 4;
    const CUtensorMapSwizzle asw = S == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : S == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                   : S == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
    return encode_tiled(&w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, packed, wdims, wstr, wbox,
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_tiled(&am, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, absmax, adims, astr, abox, asw);
  };
  if (!maps(wgu, agu, a.gu_packed, a.gu_absmax, n1, a.H) || !maps(wdn, adn, a.dn_packed, a.dn_absmax, a.H, a.I))
    return E4B_ERR_CUDA;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(decode_layer_grid());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = DSmem::total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, wgu, agu, wdn, adn) != cudaSuccess) return E4B_ERR_CUDA;
  return launch_status();
}


template <typename OutT, int PW>
static e4b_status launch_slice(const DecodeArgs& a, cudaStream_t s) {
  static unsigned long long configured = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return E4B_ERR_CUDA;
  const unsigned long long bit = 1ull << dev;
  auto kern = nf4_decode_slice_kernel<OutT, PW>;
  {
    std::lock_guard<std::mutex> lk(g_dl_mu);
    if (!(configured & bit)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, DSmem::total) != cudaSuccess)
        return E4B_ERR_CUDA;
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, DSmem::total) != cudaSuccess ||
          per_sm < 1)
        return E4B_ERR_UNSUPPORTED;
      configured |= bit;
    }
  }
  CUtensorMap gw, ga, dw, da;
  // The four maps depend only on the stacks' addresses and the layer geometry: a small cache per
  // device (a model's layers, round robin) saves their encoding on every decode step.
  struct MapSet {
    const void* p[4];
    int E, H, I;
    CUtensorMap m[4];
  };
  constexpr int kMapSets = 64;
  static MapSet* map_cache[64] = {nullptr};
  static int map_next[64] = {0};
  const void* keys[4] = {a.gu_packed, a.gu_absmax, a.dn_packed, a.dn_absmax};
  bool cached = false;
  {
    std::lock_guard<std::mutex> lk(g_dl_mu);
    if (MapSet* c = map_cache[dev]) {
      for (int i = 0; i < kMapSets && !cached; ++i) {
        const MapSet& ms = c[i];
        if (ms.p[0] == keys[0] && ms.p[1] == keys[1] && ms.p[2] == keys[2] && ms.p[3] == keys[3] && ms.E == a.E &&
            ms.H == a.H && ms.I == a.I) {
          gw = ms.m[0];
          ga = ms.m[1];
          dw = ms.m[2];
          da = ms.m[3];
          cached = true;
        }
      }
    }
  }
  const cuuint64_t gu_rows = (cuuint64_t)a.E * 2 * a.I, dn_rows = (cuuint64_t)a.E * a.H;
  if (!cached) {
  {  // gate_up packed as [lines (H / 256)][rows][128 B]; a box is 2 lines x 64 rows
    const cuuint64_t dims[3] = {128, gu_rows, (cuuint64_t)(a.H / 256)};
    const cuuint64_t str[2] = {(cuuint64_t)(a.H / 2), 128};
    const cuuint32_t box[3] = {128, 64, 2};
    if (!encode_tiled(&gw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a.gu_packed, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return E4B_ERR_CUDA;
  }
  {  // gate_up absmax [rows][H / 64]; a box is 8 blocks x 64 rows
    const cuuint64_t dims[2] = {(cuuint64_t)(a.H / 64), gu_rows};
    const cuuint64_t str[1] = {(cuuint64_t)(a.H / 64) * 4};
    const cuuint32_t box[2] = {8, 64};
    if (!encode_tiled(&ga, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.gu_absmax, dims, str, box, CU_TENSOR_MAP_SWIZZLE_32B))
      return E4B_ERR_CUDA;
  }
  {  // down packed [rows][I / 2]; a box is one 32-byte block column x 256 rows
    const cuuint64_t dims[2] = {(cuuint64_t)(a.I / 2), dn_rows};
    const cuuint64_t str[1] = {(cuuint64_t)(a.I / 2)};
    const cuuint32_t box[2] = {32, 256};
    if (!encode_tiled(&dw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a.dn_packed, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return E4B_ERR_CUDA;
  }
  {  // down absmax [rows][I / 64]; a box is 4 blocks x 256 rows
    const cuuint64_t dims[2] = {(cuuint64_t)(a.I / 64), dn_rows};
    const cuuint64_t str[1] = {(cuuint64_t)(a.I / 64) * 4};
    const cuuint32_t box[2] = {4, 256};
    if (!encode_tiled(&da, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.dn_absmax, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return E4B_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_dl_mu);
  if (!map_cache[dev]) map_cache[dev] = new (std::nothrow) MapSet[kMapSets]();
  if (MapSet* c = map_cache[dev]) {
    MapSet& ms = c[map_next[dev]];
    map_next[dev] = (map_next[dev] + 1) % kMapSets;
    for (int i = 0; i < 4; ++i) ms.p[i] = keys[i];
    ms.E = a.E;
    ms.H = a.H;
    ms.I = a.I;
    ms.m[0] = gw;
    ms.m[1] = ga;
    ms.m[2] = dw;
    ms.m[3] = da;
  }
  }
  // The fused router runs over the whole grid through global scratch, or (on request) in clusters
  // of 4 (or 2) CTAs when a grid of co-resident clusters covers (nearly) every SM and the device
  // takes the clustered cooperative launch.
  int grid = decode_layer_grid(), cs = 1;
  if (a.router_w) {
    std::lock_guard<std::mutex> lk(g_dl_mu);
    static int cl_size[64] = {0}, cl_grid[64] = {0};
    if (!cl_size[dev]) {
      int best_cs = 1, best_grid = grid;
      for (int c : {4, 2}) {
        cudaLaunchConfig_t q{};
        q.gridDim = dim3(grid / c * c);
        q.blockDim = dim3(kThreads);
        q.dynamicSmemBytes = DSmem::total;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = c;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        int ncl = 0;
        if (cudaOccupancyMaxActiveClusters(&ncl, kern, &q) != cudaSuccess) {
          cudaGetLastError();
          continue;
        }
        const int g = ncl * c < grid / c * c ? ncl * c : grid / c * c;
        if (g * 20 >= grid * 19) {  // within 5 % of the full grid
          best_cs = c;
          best_grid = g;
          break;
        }
      }
      cl_size[dev] = best_cs;
      cl_grid[dev] = best_grid;
    }
    // clusters only on request (E4B_SLICE_CLUSTER=1): every CTA then runs logit tasks before its
    // own set-up, which measured slower than the grid-wide split on the OLMoE decode step
    static const bool no_cluster = [] {
      const char* v = getenv("E4B_SLICE_CLUSTER");
      return !(v && v[0] == '1');
    }();
    cs = (no_cluster || g_slice_no_cluster[dev].load()) ? 1 : cl_size[dev];
    if (cs > 1) grid = cl_grid[dev];
  }
  // stage hand-off (E4B_SLICE_FLAGS): both bits by default, 2 % faster at T=1 and 3-6 % at T=4
  // on the OLMoE step than a per-warp fence and a waiting producer
  static const int flags = [] {
    const char* v = getenv("E4B_SLICE_FLAGS");
    return v ? atoi(v) & 3 : 3;
  }();
  for (;;) {
    DecodeArgs la = a;
    la.cluster = cs;
    la.slice_flags = flags;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = DSmem::total;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    int na = 1;
    if (cs > 1) {
      attr[1].id = cudaLaunchAttributeClusterDimension;
      attr[1].val.clusterDim.x = cs;
      attr[1].val.clusterDim.y = 1;
      attr[1].val.clusterDim.z = 1;
      na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, la, gw, ga, dw, da);
    if (e == cudaSuccess) break;
    if (cs == 1) return E4B_ERR_CUDA;
    cudaGetLastError();  // clustered cooperative launch refused: the grid-wide router from now on
    cs = 1;
    grid = decode_layer_grid();
    slice_cluster_off(dev);
  }
  return launch_status();
}

e4b_status launch_decode_layer(const e4b_moe_desc& d, const e4b_moe_tensors* t, void* h, void* down_rows,
                               void* sync, int* err, cudaStream_t s, const DecodeRouter* router, void* part) {
  DecodeArgs a{};
  if (router) {
    a.router_w = router->weight;
    a.router_w_dtype = router->weight_dtype;
    a.route_kind = router->kind;
    a.renorm = router->norm_topk_prob;
    a.topk_idx_out = router->topk_idx;
    a.topk_w_out = router->topk_w;
    a.router_logits = router->logits;
  }
  a.hidden = t->hidden;
  a.act_dtype = d.act_dtype;
  a.topk_idx = t->topk_idx;
  a.topk_w = t->topk_w;
  a.emap = t->expert_map;
  a.routed = d.routed_experts;
  a.w_dtype = router ? E4B_F32 : d.weight_dtype;
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
  a.down_rows = static_cast<__half*>(down_rows);
  a.cta_err = static_cast<int*>(sync);
  a.err = err;
  if (part && decode_mode() == 3 && decode_slice_shape(d)) {
    a.part = static_cast<float*>(part);
    // words of each block decoded in registers instead of the shared pair table (E4B_SLICE_PW;
    // 0 by default: on the OLMoE decode step 1 and 2 measured 3 % and 7 % slower -- the streaming
    // loop is latency-bound, not bound by the shared-memory pipe)
    static const int pw = [] {
      const char* v = getenv("E4B_SLICE_PW");
      return v ? (v[0] == '1' ? 1 : v[0] == '2' ? 2 : 0) : 0;
    }();
#define E4B_SLICE_LAUNCH(P)                                                   \
  switch (d.out_dtype) {                                                      \
    case E4B_BF16: return launch_slice<__nv_bfloat16, P>(a, s);               \
    case E4B_F16: return launch_slice<__half, P>(a, s);                       \
    default: return launch_slice<float, P>(a, s);                             \
  }
    if (pw == 1) E4B_SLICE_LAUNCH(1)
    if (pw == 2) E4B_SLICE_LAUNCH(2)
    E4B_SLICE_LAUNCH(0)
#undef E4B_SLICE_LAUNCH
  }
  const bool two = d.tokens > 8;
  switch (d.out_dtype) {
    case E4B_BF16: return two ? launch_decode<__nv_bfloat16, 2>(a, s) : launch_decode<__nv_bfloat16, 1>(a, s);
    case E4B_F16: return two ? launch_decode<__half, 2>(a, s) : launch_decode<__half, 1>(a, s);
    default: return two ? launch_decode<float, 2>(a, s) : launch_decode<float, 1>(a, s);
  }
}

}  // namespace e4b

extern "C" E4B_API int e4b_set_decode_kernel(int mode) {
  const int prev = e4b::decode_mode();
  e4b::g_decode_mode.store(mode == 0 ? 0 : mode == 1 ? 1 : mode == 2 ? 2 : 3);
  return prev;
}
