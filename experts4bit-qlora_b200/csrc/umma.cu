// tcgen05 grouped NF4 GEMM for the prefill regime (many tokens per expert).
//
// Replaces grouped-nf4-gemm's gemm_4bit_grouped at prefill shapes
// (experts4bit_qlora/engines/fast.py:137-156) with the gate_up epilogue
// (lora._epilogue, lora.py:102-128) and the LoRA delta (lora.py:251-256) fused.
//
// D[token, feature] = X[token, :] . W_e[feature, :] on the 5th-generation tensor
// cores: a tile of 128 tokens of one expert is the M = 128 operand, the tile's
// decoded weight rows the N operand, fp32 accumulators live in tensor memory.
// For SwiGLU the CTA tile is 128 output features: its 128 gate rows and the 128
// matching up rows form one N = 256 operand, so one MMA per k-step covers both
// and silu(gate) * up happens in the thread that owns the token.
//
// One persistent CTA per SM, 24 warps with fixed roles, 64-wide K chunks (one
// quantization block per row per chunk) through three rings of their own depth --
// packed weights 4 deep, activation tiles 3 deep, decoded weight tiles 3 deep:
//   warp 0      TMA: packed NF4 bytes of the tile's rows (2-D boxes {32 B, 128 rows}, 32-byte
//               swizzle);
//   warp 1      TMA of the 128 token rows (fp16, expert-sorted), one box per chunk,
//               landing in the 128-byte-swizzled K-major operand layout;
//   warp 3      allocates TMEM, issues tcgen05.mma (one thread), commits;
//   warps 4-19  NF4 -> fp16 decode: two threads per weight row, each 16 pair-table
//               lookups per chunk (its half of the row's 64 elements), scaled by the
//               block's absmax, stored into the swizzled, K-major weight operand;
//   warps 20-23 epilogue: tcgen05.ld of the finished accumulators (double
//               buffered, so it overlaps the next tile's MMAs), one token row per
//               thread: activation scale, activation, 16-byte stores.
// With an adapter, each tile takes one more chunk: the activation warp loads the
// tile's LoRA-A products (fp16, from the LoRA-A pre-pass), the decode warps write
// the LoRA-B rows of the tile's features, and the MMA adds a K = 16 step, so the
// delta enters the accumulator on the tensor cores (before the activation, as
// lora.py:102-128 adds it).
// Tiles are ordered (expert, feature tile, token tile) so CTAs that run at the
// same time share the weight tile through L2. Every wait is bounded; a timeout
// raises E4B_ERR_TIMEOUT and all roles run to the common exit (TMEM is freed).
#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "async.cuh"
#include "fp8.cuh"
#include "umma.cuh"
#include "tmap.cuh"
#include "nf4_prmt.cuh"

// Profiling instrumentation, compiled only with -DE4B_TRACE: per-CTA cycles each role
// spends waiting (clock64), read back with e4b_umma_stats_read.
#ifdef E4B_TRACE
__device__ unsigned long long g_umma_stats[148 * 16];
extern "C" __attribute__((visibility("default"))) int e4b_umma_stats_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, g_umma_stats, sizeof(g_umma_stats));
}
#define STAT_WAIT(slot, expr)                                                        \
  ({                                                                                 \
    const long long t0_ = clock64();                                                 \
    const bool ok_ = (expr);                                                         \
    if (blockIdx.x < 148) atomicAdd(&g_umma_stats[blockIdx.x * 16 + (slot)], (unsigned long long)(clock64() - t0_)); \
    ok_;                                                                             \
  })
#else
#define STAT_WAIT(slot, expr) (expr)
#endif

namespace e4b {

namespace {

constexpr int kSW = 3;  // packed-weight ring depth (HBM latency)
constexpr int kSB = 4;  // activation ring depth
constexpr int kSA = 3;  // decoded-weight ring depth: the decode runs up to two chunks ahead of the MMA
constexpr int kTok = kUmmaTokens;  // 128 tokens per tile (UMMA M)
constexpr int kRows = 128;          // weight rows per group (UMMA M)
constexpr int kKc = 64;             // K per chunk
constexpr int kThreads = 512;     // dgrad kernel: 4 control warps, 8 decode warps, 4 epilogue warps
constexpr int kDec = 512;         // forward kernel: decode threads (two per weight row)
constexpr int kFwdThreads = 128 + kDec + 128;  // forward kernel: control, decode, epilogue warps
constexpr int kABytes = kRows * kKc * 2;        // 16 KB fp16 per group
constexpr int kBBytes = kTok * kKc * 2;         // 16 KB fp16
constexpr int kLut = 256 * 128;
constexpr int kEpiMaxRank = 16;  // LoRA ranks above this take the streaming path

// Shared-memory plan per weight format: NF4 rows carry 32 packed bytes per 64-wide
// chunk and need the 32 KB pair table; FP8 rows carry 64 bytes and no table.
template <int FMT>
struct SmemT {
  static constexpr int wrow = FMT == E4B_FMT_FP8_BLOCK128 ? kKc : kKc / 2;  // weight bytes per row per chunk
  static constexpr int wbytes = kRows * wrow;                      // per group per stage
  static constexpr int lut = 0;
  static constexpr int a = FMT == E4B_FMT_FP8_BLOCK128 ? 0 : kLut;  // [stage][group] 16 KB, 1024-aligned
  static constexpr int b = a + kSA * 2 * kABytes;                 // [stage] 16 KB
  static constexpr int w = b + kSB * kBBytes;                     // [stage][group]
  static constexpr int epi = w + kSW * 2 * wbytes;                // epilogue staging
  static constexpr int bars = epi;
  // full_w, w_empty [kSW]; full_b, b_empty [kSB]; a_ready, a_empty [kSA]; acc_full, acc_empty [2]
  static constexpr int nbars = 2 * kSW + 2 * kSB + 2 * kSA + 4;
  static constexpr int tmem_slot = bars + nbars * 8;
  static constexpr int tables = tmem_slot + 16;                   // tile_start and offsets, E <= 1024
  static constexpr int total = tables + 2 * 1025 * 4;
};

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity);

// Bounded wait that remembers a timeout: after the first timeout every later
// wait of this thread returns at once, so all roles reach the common exit.
struct Waiter {
  bool dead = false;
  int* err;
  __device__ bool wait(uint64_t* bar, uint32_t parity) {
    if (dead) return false;
    if (mbar_wait(bar, parity)) return true;
    dead = true;
    raise_error(err, E4B_ERR_TIMEOUT);
    return false;
  }
  // the same with cluster-scope acquire, for barriers the other CTA of a pair arrives on
  __device__ bool waitc(uint64_t* bar, uint32_t parity) {
    if (dead) return false;
    for (uint32_t i = 0; i < kMaxSpins; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    dead = true;
    raise_error(err, E4B_ERR_TIMEOUT);
    return false;
  }
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzle shared-memory matrix descriptor (rows of 128 B, 8-row groups 1024 B apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fff);          // start address
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                          // descriptor version
  d |= (uint64_t)2 << 61;                          // layout: 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: fp16 (or, with bf16, bf16) A and B, fp32 D, both K-major,
// M = 128 tokens, N = n features.
__device__ __forceinline__ uint32_t idesc_f16(int n, bool bf16 = false) {
  const uint32_t ab = bf16 ? (1u << 7) | (1u << 10) : 0u;
  return (1u << 4) | ab | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTok >> 4) << 24);
}

// e2m1 values (OCP microscaling FP4), index = 4-bit code
__constant__ float c_e2m1_umma[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                      -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

// 2^(s-127) as bf16 bits: exponent field s for s >= 1 (255: inf), subnormal 2^-127 for s = 0.
__device__ __forceinline__ uint32_t e8m0_bf16x2(uint32_t s) {
  const uint32_t b = s ? (s << 7) : 0x0040u;
  return b | (b << 16);
}

__device__ __forceinline__ void umma_f16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- CTA-pair (cta_group::2) helpers: the even CTA of a cluster of two issues the MMA ----------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `p`'s counterpart in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Tiled TMA load (no multicast) into this CTA's shared memory whose completion counts on the
// barrier at `bar_caddr` (shared::cluster), which may be the even CTA's.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* map, int c0, int c1, uint32_t bar_caddr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(bar_caddr)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
// Arrive (once) on the barrier at `bar_caddr` when the pair's MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_caddr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_caddr)
               : "memory");
}

// silu for the accumulator epilogue: the quotient with the fast approximate divide (a reciprocal
// and a multiply, about 2 ulp of fp32) instead of the IEEE division sequence; the result is then
// rounded to the 16-bit output type, far coarser. For x below about -87, exp(-x) overflows and the
// quotient is 0 (the exact value is below 1e-36 in magnitude).
__device__ __forceinline__ float silu_epi(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// First weight row of group h of feature tile ft. SwiGLU: the tile's 128 gate rows and the
// matching 128 up rows; otherwise (GROUPS == 2) 256 consecutive rows, (GROUPS == 1) 128.
__device__ __forceinline__ int group_row0(const GemvArgs& g, int ft, int h, int groups) {
  if (g.epilogue == E4B_EPI_SWIGLU) return h == 0 ? ft * 128 : (g.N / 2) + ft * 128;
  return ft * 128 * groups + h * 128;
}

struct TileInfo {
  int e, row0, M, ft, tt;
};

// Tile t -> (expert, token tile, feature tile); tiles ordered (expert, feature tile, token tile).
// ts (prefix of ceil(count / kTok)) and offs are the shared-memory copies of the expert tables.
__device__ __forceinline__ void tile_info(const int32_t* ts, const int32_t* offs, int E, int nft, int t,
                                          TileInfo& ti) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {  // last e with ts[e] * nft <= t
    const int mid = (lo + hi + 1) >> 1;
    if (ts[mid] * nft <= t) lo = mid; else hi = mid - 1;
  }
  ti.e = lo;
  const int local = t - ts[lo] * nft;
  const int ntt = ts[lo + 1] - ts[lo];
  ti.ft = local / ntt;
  ti.tt = local - ti.ft * ntt;
  ti.row0 = offs[lo];
  ti.M = offs[lo + 1] - ti.row0;
}

}  // namespace

static_assert(SmemT<E4B_FMT_NF4>::total <= 232448 && SmemT<E4B_FMT_FP8_BLOCK128>::total <= 232448,
              "shared memory budget");

// PAIR (NF4, GROUPS == 2): clusters of two CTAs run tcgen05.mma.cta_group::2 with M = 256 tokens
// (128 per CTA) and N = 256 features. Each CTA decodes only its own group of 128 weight rows
// (four decode threads per row) and loads its own 128 token rows, so per MMA FLOP a CTA decodes
// half as many weights and its shared memory serves half the weight operand. The even CTA issues
// the MMAs, waits on both CTAs' operands (TMA completion and decode warps arrive on its barriers)
// and commits to the barriers of both; each CTA's epilogue reads its own 128 TMEM lanes.
template <typename OutT, int GROUPS, int FMT, bool PAIR = false>
__global__ void __launch_bounds__(kFwdThreads, 1)
    nf4_umma_kernel(UmmaArgs u, const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap bmap,
                    const __grid_constant__ CUtensorMap lmap) {
  using Smem = SmemT<FMT>;
  constexpr int kWBytes = Smem::wbytes;
  extern __shared__ __align__(1024) char smem[];
#ifdef E4B_TRACE
  const long long t_start = clock64();
#endif
  const GemvArgs& g = u.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  char* lut = smem + Smem::lut;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::bars);
  uint64_t* full_w = bars;
  uint64_t* w_empty = full_w + kSW;
  uint64_t* full_b = w_empty + kSW;
  uint64_t* b_empty = full_b + kSB;
  uint64_t* a_ready = b_empty + kSB;
  uint64_t* a_empty = a_ready + kSA;
  uint64_t* acc_full = a_empty + kSA;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Smem::tmem_slot);
  int32_t* s_ts = reinterpret_cast<int32_t*>(smem + Smem::tables);
  int32_t* s_offs = s_ts + 1025;
  for (int i = tid; i <= u.g.E; i += kFwdThreads) {
    if (!PAIR) s_ts[i] = u.tile_start[i];
    s_offs[i] = u.g.offsets[i];
  }
  const uint32_t crank = PAIR ? cluster_rank() : 0;  // PAIR: 0 issues the MMAs
  if (PAIR && warp == 2) {  // token-pair tiles: prefix of ceil(count / 256) per expert
    int carry = 0;
    for (int base = 0; base < u.g.E; base += 32) {
      const int e = base + lane;
      const int v = e < u.g.E ? (u.g.offsets[e + 1] - u.g.offsets[e] + 2 * kTok - 1) / (2 * kTok) : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (e < u.g.E) s_ts[e + 1] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_ts[0] = 0;
  }
  // work units: tiles (one CTA) or token-pair tiles (one cluster of two)
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int unit_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  const int nft = g.N / (GROUPS * kRows);  // feature tiles per expert (SwiGLU: gate+up rows per tile)
  const int kchunks = g.K / kKc;
  Waiter wt{false, g.err};

  if (tid == 0) {
    for (int s = 0; s < kSW; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&w_empty[s], kDec);
    }
    for (int s = 0; s < kSB; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kSA; ++s) {
      // PAIR: the even CTA's barrier also takes one arrival forwarded from the odd CTA's
      mbar_init(&a_ready[s], PAIR && crank == 0 ? kDec + 1 : kDec);
      mbar_init(&a_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], PAIR ? 8 : 128);  // PAIR: one arrival per epilogue warp of each CTA
    }
    fence_proxy_async();
    if (PAIR) asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 3) {  // 512 TMEM columns: two buffers x (gate, up) x 128 fp32 columns
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  if (FMT == E4B_FMT_NF4) {  // pair table: entry e of lane l at (e << 7) | (l << 2)
    const float code = c_nf4[lane & 15];
    for (int e = warp; e < 256; e += kFwdThreads / 32) {
      const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
    }
  } else if (FMT == E4B_FMT_MXFP4) {  // bf16 pair table, LOW nibble first (formats/mxfp4.py:87-88)
    const float code = c_e2m1_umma[lane & 15];
    for (int e = warp; e < 256; e += kFwdThreads / 32) {
      const float first = __shfl_sync(0xffffffffu, code, e & 15), second = __shfl_sync(0xffffffffu, code, e >> 4);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__nv_bfloat16>(first, second);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // the other CTA's barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total_tiles = s_ts[g.E] * nft;

#ifdef E4B_TRACE
  const bool mma_only = !PAIR && (u.nf4_regs & 16);
#else
  constexpr bool mma_only = false;
#endif
  if (mma_only && warp != 3 && warp < 4 + kDec / 32) {
    // trace builds only: producers and decode idle
  } else if (warp == 0) {
    // ---------------- TMA producer: packed weight rows -------------------------------------
    if (lane == 0) {
      int n = 0;
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step) {
        TileInfo ti;
        tile_info(s_ts, s_offs, g.E, nft, t, ti);
        for (int c = 0; c < kchunks; ++c, ++n) {
          const int s = n % kSW;
          if (!STAT_WAIT(0, wt.wait(&w_empty[s], ((n / kSW) & 1) ^ 1))) break;
          if (PAIR) {  // this CTA's group only
            mbar_arrive_expect_tx(&full_w[s], kWBytes);
            const int row = ti.e * g.N + group_row0(g, ti.ft, (int)crank, GROUPS);
            tma_load_2d(smem + Smem::w + (s * 2) * kWBytes, &wmap, c * Smem::wrow, row, &full_w[s]);
            continue;
          }
          mbar_arrive_expect_tx(&full_w[s], GROUPS * kWBytes);
#pragma unroll
          for (int h = 0; h < GROUPS; ++h) {
            const int row = ti.e * g.N + group_row0(g, ti.ft, h, GROUPS);
            tma_load_2d(smem + Smem::w + (s * 2 + h) * kWBytes, &wmap, c * Smem::wrow, row, &full_w[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- activation tiles: one TMA box {64 halves, 128 rows} per chunk ------------
    // The rows of an expert are contiguous (expert-sorted activations); rows past its end belong
    // to the next expert or are zero-filled past the matrix, and are discarded by the epilogue.
    if (lane == 0) {
      int n = 0;
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step) {
        TileInfo ti;
        tile_info(s_ts, s_offs, g.E, nft, t, ti);
        for (int c = 0; c < kchunks + (g.rank ? 1 : 0); ++c, ++n) {  // + the tile's LoRA-A chunk
          const int s = n % kSB;
          if (!STAT_WAIT(1, wt.wait(&b_empty[s], ((n / kSB) & 1) ^ 1))) break;
          if (PAIR) {  // both CTAs' boxes complete on the even CTA's barrier
            const int trow = ti.row0 + ti.tt * 2 * kTok + (int)crank * kTok;
            const uint32_t fb = cluster_addr(&full_b[s], 0);
            if (crank == 0) mbar_arrive_expect_tx(&full_b[s], 2 * kBBytes);
            if (c < kchunks)
              tma_load_2d_pair(smem + Smem::b + s * kBBytes, &bmap, c * kKc, trow, fb);
            else
              tma_load_2d_pair(smem + Smem::b + s * kBBytes, &lmap, 0, trow, fb);
            continue;
          }
          mbar_arrive_expect_tx(&full_b[s], kBBytes);
          if (c < kchunks)
            tma_load_2d(smem + Smem::b + s * kBBytes, &bmap, c * kKc, ti.row0 + ti.tt * kTok, &full_b[s]);
          else  // scaling * (x . A^T) of the tile's tokens, fp16 rows padded to 64 columns
            tma_load_2d(smem + Smem::b + s * kBBytes, &lmap, 0, ti.row0 + ti.tt * kTok, &full_b[s]);
        }
      }
    }
  } else if (warp == 2) {
    // PAIR, odd CTA: forward each completed decoded-weight stage to the even CTA's a_ready with
    // one cluster-scope release (decode threads arrive locally, so their own loads in flight are
    // not drained by a cluster-scope release per chunk)
    if (PAIR && crank == 1 && lane == 0) {
      int n = 0;
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step)
        for (int c = 0; c < kchunks + (g.rank ? 1 : 0); ++c, ++n) {
          const int sa = n % kSA;
          if (!wt.wait(&a_ready[sa], (n / kSA) & 1)) break;
          mbar_arrive_remote(cluster_addr(&a_ready[sa], 0));
        }
    }
  } else if (warp == 3) {
    // ---------------- MMA issuer -------------------------------------------------------------
    if (PAIR && lane == 0 && crank == 0) {
      // M = 256: the A operand's rows 0..127 are this CTA's token tile, 128..255 the other CTA's
      // (same shared-memory offsets); N = 256: rows 0..127 of B from this CTA's decoded group,
      // 128..255 from the other CTA's. Each CTA's TMEM receives its own 128 token rows.
      const uint32_t idesc = (1u << 4) | ((uint32_t)((GROUPS * kRows) >> 3) << 17) | ((uint32_t)((2 * kTok) >> 4) << 24);
      int n = 0, it = 0;
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step, ++it) {
        const int buf = it & 1;
        if (!STAT_WAIT(4, wt.waitc(&acc_empty[buf], ((it >> 1) & 1) ^ 1))) break;
        tc_fence_after();
        for (int c = 0; c < kchunks + (g.rank ? 1 : 0); ++c, ++n) {
          const int s = n % kSB, sa = n % kSA;
          if (!STAT_WAIT(2, wt.waitc(&full_b[s], (n / kSB) & 1))) break;
          if (!STAT_WAIT(3, wt.waitc(&a_ready[sa], (n / kSA) & 1))) break;
          tc_fence_after();
          const uint32_t xsm = smem_u32(smem + Smem::b + s * kBBytes);
          const uint32_t wsm = smem_u32(smem + Smem::a + (sa * 2) * kABytes);
          const int ksteps = c < kchunks ? kKc / 16 : 1;
          for (int kk = 0; kk < ksteps; ++kk)
            umma_f16_pair(tmem + buf * 256, sw128_desc(xsm + kk * 32), sw128_desc(wsm + kk * 32), idesc,
                          (c | kk) != 0);
          umma_commit_pair(cluster_addr(&b_empty[s], 0));
          umma_commit_pair(cluster_addr(&b_empty[s], 1));
          umma_commit_pair(cluster_addr(&a_empty[sa], 0));
          umma_commit_pair(cluster_addr(&a_empty[sa], 1));
        }
        umma_commit_pair(cluster_addr(&acc_full[buf], 0));
        umma_commit_pair(cluster_addr(&acc_full[buf], 1));
      }
    } else if (!PAIR && lane == 0) {
      const uint32_t idesc = idesc_f16(GROUPS * kRows, FMT == E4B_FMT_MXFP4);  // N = the tile's gate (+ up) rows
      int n = 0, it = 0;
#ifdef E4B_TRACE
      if (u.nf4_regs & 16) {  // trace builds only: MMAs on whatever the first ring slots hold, no operand waits
        for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step, ++it) {
          const int buf = it & 1;
          if (!STAT_WAIT(4, wt.wait(&acc_empty[buf], ((it >> 1) & 1) ^ 1))) break;
          tc_fence_after();
          for (int c = 0; c < kchunks; ++c) {
            if (u.nf4_regs & 64) {  // a completed barrier's wait and the fence, as the fed loop does
              if (!STAT_WAIT(2, wt.wait(&full_w[0], 1))) break;
              tc_fence_after();
            }
            const uint32_t xsm = smem_u32(smem + Smem::b + (c % kSB) * kBBytes);
            const uint32_t wsm = smem_u32(smem + Smem::a + ((c % kSA) * 2) * kABytes);
            for (int kk = 0; kk < kKc / 16; ++kk)
              umma_f16(tmem + buf * 256, sw128_desc(xsm + kk * 32), sw128_desc(wsm + kk * 32), idesc, (c | kk) != 0);
            if (u.nf4_regs & 32) umma_commit(&b_empty[0]);  // commit cost, barrier unused in this mode
          }
          umma_commit(&acc_full[buf]);
        }
      } else
#endif
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step, ++it) {
        const int buf = it & 1;
        if (!STAT_WAIT(4, wt.wait(&acc_empty[buf], ((it >> 1) & 1) ^ 1))) break;
        tc_fence_after();
        for (int c = 0; c < kchunks + (g.rank ? 1 : 0); ++c, ++n) {  // + the LoRA chunk (one K = 16 step)
          const int s = n % kSB, sa = n % kSA;
          if (!STAT_WAIT(2, wt.wait(&full_b[s], (n / kSB) & 1))) break;
          if (!STAT_WAIT(3, wt.wait(&a_ready[sa], (n / kSA) & 1))) break;
          tc_fence_after();
          // D[token][feature] += X[token][k] . W[feature][k]: the 128 tokens are the M operand, the
          // tile's decoded gate and up rows (adjacent 16 KB groups) one N = 256 operand
          const uint32_t xsm = smem_u32(smem + Smem::b + s * kBBytes);
          const uint32_t wsm = smem_u32(smem + Smem::a + (sa * 2) * kABytes);
          const int ksteps = c < kchunks ? kKc / 16 : 1;
          for (int kk = 0; kk < ksteps; ++kk)
            umma_f16(tmem + buf * 256, sw128_desc(xsm + kk * 32), sw128_desc(wsm + kk * 32), idesc, (c | kk) != 0);
          umma_commit(&b_empty[s]);
          umma_commit(&a_empty[sa]);
        }
        umma_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 4 + kDec / 32) {
    // ---------------- decode: two threads per weight row, each half of the row's chunk -------
    const int d = tid - 128;            // 0..kDec-1
    const int part = d >> 8;            // 0: elements 0..31 of the chunk, 1: elements 32..63
    const int h = (d >> 7) & 1, r = d & 127;  // group, row within the tile
    const uint32_t lane4 = (uint32_t)lane << 2;
    const Nf4Bytes nfb = nf4_bytes();
    int nw = 0, na = 0;  // packed-weight ring items, decoded-weight ring items (the LoRA chunk has no packed weights)
    // LoRA chunk of a tile: this row's LoRA-B values (rank <= 16, fp16) as K elements 0..15 of the
    // weight operand; the MMA issues a single K = 16 step for it, so the rest of the row is unused.
    auto lora_chunk = [&](const TileInfo& ti, int row) -> bool {
      const int sa = na % kSA;
      if (!wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1)) return false;
      if (h < GROUPS) {  // part p writes unit p: the row's LoRA-B values 8p .. 8p+7
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = 8 * part + j < g.rank
                     ? load_as_f32(g.lora_B, g.lora_dtype, ((int64_t)ti.e * g.N + row) * g.rank + 8 * part + j)
                     : 0.f;
        char* adst = smem + Smem::a + (sa * 2 + h) * kABytes + r * 128;
        const int swz = (smem_u32(adst) >> 7) & 7;
        *reinterpret_cast<uint4*>(adst + ((part ^ swz) << 4)) =
            make_uint4(pack2<__half>(v[0], v[1]), pack2<__half>(v[2], v[3]), pack2<__half>(v[4], v[5]),
                       pack2<__half>(v[6], v[7]));
      }
      fence_proxy_async();
      mbar_arrive(&a_ready[sa]);
      ++na;
      return true;
    };
    if constexpr (PAIR) {
      // Four threads per weight row of this CTA's group: lane l of decode warp w owns row
      // 8w + l / 4 and elements 16q .. 16q+15 of each chunk, q = l % 4 (packed bytes 8q .. 8q+7,
      // operand units 2q, 2q+1). Waits are warp-uniform: the warp arrives once on the even CTA's
      // a_ready after its lanes' stores and proxy fences.
      const int q = lane & 3;
      const int pr = ((d >> 5) << 3) | (lane >> 2);
      auto wok = [&](bool ok) {
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) wt.dead = true;
        return ok;
      };
      auto load_half = [&](int slot) {
        const char* wsrc = smem + Smem::w + (slot * 2) * kWBytes + pr * 32;
        const int sw = (pr >> 2) & 1;  // the 32-byte swizzle of the box
        return *reinterpret_cast<const uint2*>(wsrc + (((q >> 1) ^ sw) << 4) + ((q & 1) << 3));
      };
      for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step) {
        TileInfo ti;
        tile_info(s_ts, s_offs, g.E, nft, t, ti);
        const int row = group_row0(g, ti.ft, (int)crank, GROUPS) + pr;
        const float* am = g.absmax + ((int64_t)ti.e * g.N + row) * (g.K / 64);
        // absmax four chunks at a time, the next four loaded one group ahead
        const bool vec4 = (g.K & 255) == 0;
        auto load4 = [&](int c0) {
          if (vec4) return __ldg(reinterpret_cast<const float4*>(am + c0));
          float4 v;
          v.x = __ldg(am + c0);
          v.y = c0 + 1 < kchunks ? __ldg(am + c0 + 1) : 0.f;
          v.z = c0 + 2 < kchunks ? __ldg(am + c0 + 2) : 0.f;
          v.w = c0 + 3 < kchunks ? __ldg(am + c0 + 3) : 0.f;
          return v;
        };
        float4 am_cur = load4(0), am_nxt = kchunks > 4 ? load4(4) : am_cur;
        uint2 p_next = make_uint2(0, 0);
        for (int c = 0; c < kchunks; ++c, ++nw, ++na) {
          const int s = nw % kSW, sa = na % kSA;
          if ((c & 3) == 0 && c > 0) {
            am_cur = am_nxt;
            if (c + 4 < kchunks) am_nxt = load4(c + 4);
          }
          const float a = (c & 3) == 0 ? am_cur.x : (c & 3) == 1 ? am_cur.y : (c & 3) == 2 ? am_cur.z : am_cur.w;
          uint2 p0 = p_next;
          if (c == 0) {
            if (!wok(tid == 128 ? STAT_WAIT(5, wt.wait(&full_w[s], (nw / kSW) & 1)) : wt.wait(&full_w[s], (nw / kSW) & 1))) break;
            p0 = load_half(s);
          }
          if (c + 1 < kchunks) {  // next chunk's bytes before this chunk's decode
            const int s1 = (nw + 1) % kSW;
            if (!wok(wt.wait(&full_w[s1], ((nw + 1) / kSW) & 1))) break;
            p_next = load_half(s1);
          }
          if (!wok(wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1))) break;
          const uint32_t words[2] = {p0.x, p0.y};
          const __half2 sc = __float2half2_rn(a);
          char* adst = smem + Smem::a + (sa * 2) * kABytes + pr * 128;
          const int swz = (smem_u32(adst) >> 7) & 7;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            uint32_t o[4];
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
              const uint32_t byte = (words[j] >> (8 * bb)) & 0xffu;
              uint32_t pv = *reinterpret_cast<const uint32_t*>(lut + ((byte << 7) | lane4));
              __half2 v = __hmul2(*reinterpret_cast<__half2*>(&pv), sc);
              o[bb] = *reinterpret_cast<uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(adst + (((2 * q + j) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
          fence_proxy_async();
          mbar_arrive(&w_empty[s]);  // this thread's packed bytes were consumed above
          mbar_arrive(&a_ready[sa]);  // this CTA's barrier; the odd CTA's is forwarded (warp 2)
        }
        if (g.rank && !wt.dead) {  // LoRA-B values of the row: quarters 0, 1 write units 0, 1
          const int sa = na % kSA;
          if (!wok(wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1))) break;
          if (q < 2) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              v[j] = 8 * q + j < g.rank
                         ? load_as_f32(g.lora_B, g.lora_dtype, ((int64_t)ti.e * g.N + row) * g.rank + 8 * q + j)
                         : 0.f;
            char* adst = smem + Smem::a + (sa * 2) * kABytes + pr * 128;
            const int swz = (smem_u32(adst) >> 7) & 7;
            *reinterpret_cast<uint4*>(adst + ((q ^ swz) << 4)) =
                make_uint4(pack2<__half>(v[0], v[1]), pack2<__half>(v[2], v[3]), pack2<__half>(v[4], v[5]),
                           pack2<__half>(v[6], v[7]));
          }
          fence_proxy_async();
          mbar_arrive(&a_ready[sa]);
          ++na;
        }
      }
    } else
    for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step) {
      TileInfo ti;
      tile_info(s_ts, s_offs, g.E, nft, t, ti);
      const int row = group_row0(g, ti.ft, h, GROUPS) + r;
      if (FMT == E4B_FMT_FP8_BLOCK128) {
        // e4m3 row -> fp16(fp32(w) * s_kb / s_ref): the tile's 128 rows share one scale per 128-wide
        // K block; s_ref (the largest over K) goes back in the epilogue. For e8m0 scales the ratio
        // is a power of two <= 1 and the operand is exact while it stays above fp16's 2^-24.
        const float* sc = g.absmax + ((int64_t)ti.e * (g.N / kFp8Block) + row / kFp8Block) * (g.K / kFp8Block);
        float inv_ref = 0.f;
        if (h < GROUPS) {
          float m = 0.f;
          for (int kb = 0; kb < g.K / kFp8Block; ++kb) m = fmaxf(m, __ldg(sc + kb));
          inv_ref = m > 0.f ? 1.f / m : 0.f;
        }
        const bool pipelined = (u.nf4_regs & 6) == 6;  // next chunk's units loaded before this decode
        const int rot = r & 3;  // rotated unit order spreads a quarter-warp over the banks
        auto load_units = [&](int slot, uint4 (&q)[2]) {  // part p: the row's 16-byte units 2p, 2p+1
          if (h < GROUPS) {
            const uint4* wsrc = reinterpret_cast<const uint4*>(smem + Smem::w + (slot * 2 + h) * kWBytes + r * 64);
#pragma unroll
            for (int u4 = 0; u4 < 2; ++u4) q[u4] = wsrc[(2 * part + u4 + rot) & 3];
          }
        };
        uint4 pn[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        for (int c = 0; c < kchunks; ++c, ++nw, ++na) {
          const int s = nw % kSW, sa = na % kSA;
          const float scale = h < GROUPS ? __ldg(sc + (c >> 1)) * inv_ref : 0.f;
          uint4 p[2] = {pn[0], pn[1]};
          if (!(pipelined && c > 0)) {
            if (!(tid == 128 ? STAT_WAIT(5, wt.wait(&full_w[s], (nw / kSW) & 1)) : wt.wait(&full_w[s], (nw / kSW) & 1))) break;
            load_units(s, p);
          }
          if (pipelined && c + 1 < kchunks) {
            const int s1 = (nw + 1) % kSW;
            if (!wt.wait(&full_w[s1], ((nw + 1) / kSW) & 1)) break;
            load_units(s1, pn);
          }
          if (!(u.nf4_regs & 2)) {  // release the packed slot now (else after the decode, one fence for both)
            fence_proxy_async();  // generic reads of the slot before its refill by the async proxy
            mbar_arrive(&w_empty[s]);
          }
          if (!wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1)) break;
          if (h < GROUPS) {
            char* adst = smem + Smem::a + (sa * 2 + h) * kABytes + r * 128;
            const int swz = (smem_u32(adst) >> 7) & 7;
#pragma unroll
            for (int u4 = 0; u4 < 2; ++u4) {  // 16 weight bytes -> A units 2U, 2U+1 (8 fp16 each)
              const int U = (2 * part + u4 + rot) & 3;
              const uint32_t wd[4] = {p[u4].x, p[u4].y, p[u4].z, p[u4].w};
              uint32_t o[8];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                o[2 * j] = e4m3x2_to_f16x2_scaled(wd[j] & 0xffffu, scale);
                o[2 * j + 1] = e4m3x2_to_f16x2_scaled(wd[j] >> 16, scale);
              }
              *reinterpret_cast<uint4*>(adst + (((2 * U) ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
              *reinterpret_cast<uint4*>(adst + (((2 * U + 1) ^ swz) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            }
          }
          fence_proxy_async();
          if (u.nf4_regs & 2) mbar_arrive(&w_empty[s]);  // the packed bytes were consumed above
          mbar_arrive(&a_ready[sa]);
        }
        if (g.rank && !wt.dead) lora_chunk(ti, row);
        continue;
      }
      if (FMT == E4B_FMT_MXFP4) {
        // e2m1 pairs -> bf16 through the pair table, times the block's 2^(s-127) (exact in bf16);
        // a 64-wide chunk is two 32-element scale blocks
        const uint8_t* sp = reinterpret_cast<const uint8_t*>(g.absmax) + ((int64_t)ti.e * g.N + row) * (g.K / 32);
        const bool pipelined = (u.nf4_regs & 6) == 6;
        uint4 pn = make_uint4(0, 0, 0, 0);
        for (int c = 0; c < kchunks; ++c, ++nw, ++na) {
          const int s = nw % kSW, sa = na % kSA;
          uint32_t s0 = 0;  // part p: scale block p of the chunk (elements 32p .. 32p+31)
          if (h < GROUPS) s0 = e8m0_bf16x2(__ldg(sp + 2 * c + part));
          auto load_unit = [&](int slot) {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (h < GROUPS) {
              const char* wsrc = smem + Smem::w + (slot * 2 + h) * kWBytes + r * 32;
              const int sw = (r >> 2) & 1;  // the 32-byte swizzle of the box (rows r and r + 4 apart)
              v = reinterpret_cast<const uint4*>(wsrc)[part ^ sw];
            }
            return v;
          };
          uint4 p0 = pn;
          if (!(pipelined && c > 0)) {
            if (!wt.wait(&full_w[s], (nw / kSW) & 1)) break;
            p0 = load_unit(s);
          }
          if (pipelined && c + 1 < kchunks) {  // next chunk's unit before this chunk's decode
            const int s1 = (nw + 1) % kSW;
            if (!wt.wait(&full_w[s1], ((nw + 1) / kSW) & 1)) break;
            pn = load_unit(s1);
          }
          if (!(u.nf4_regs & 2)) {  // release the packed slot now (else after the decode, one fence for both)
            fence_proxy_async();  // generic reads of the slot before its refill by the async proxy
            mbar_arrive(&w_empty[s]);
          }
          if (!wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1)) break;
          if (h < GROUPS) {
            const uint32_t words[4] = {p0.x, p0.y, p0.z, p0.w};
            char* adst = smem + Smem::a + (sa * 2 + h) * kABytes + r * 128;
            const int swz = (smem_u32(adst) >> 7) & 7;
            const __nv_bfloat162 sc2 = *reinterpret_cast<const __nv_bfloat162*>(&s0);
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {  // unit q = elements 8q .. 8q+7
              const int q = 4 * part + qq;
              uint32_t o[4];
#pragma unroll
              for (int bb = 0; bb < 4; ++bb) {
                const uint32_t byte = (words[qq] >> (8 * bb)) & 0xffu;
                uint32_t pr = *reinterpret_cast<const uint32_t*>(lut + ((byte << 7) | lane4));
                __nv_bfloat162 v = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&pr), sc2);
                o[bb] = *reinterpret_cast<uint32_t*>(&v);
              }
              *reinterpret_cast<uint4*>(adst + ((q ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
          fence_proxy_async();
          if (u.nf4_regs & 2) mbar_arrive(&w_empty[s]);  // the packed bytes were consumed above
          mbar_arrive(&a_ready[sa]);
        }
        continue;
      }
      const float* am = g.absmax + ((int64_t)ti.e * g.N + row) * (g.K / 64);
      // absmax four chunks at a time (one 16-byte load when K % 256 == 0 keeps it aligned, else
      // four scalar loads), the next group loaded one group ahead so its latency hides behind four
      // chunks of decode
      const bool vec4 = (g.K & 255) == 0;
      auto load4 = [&](int c0) {
        if (vec4) return __ldg(reinterpret_cast<const float4*>(am + c0));
        float4 v;
        v.x = __ldg(am + c0);
        v.y = c0 + 1 < kchunks ? __ldg(am + c0 + 1) : 0.f;
        v.z = c0 + 2 < kchunks ? __ldg(am + c0 + 2) : 0.f;
        v.w = c0 + 3 < kchunks ? __ldg(am + c0 + 3) : 0.f;
        return v;
      };
      float4 am_cur = make_float4(0.f, 0.f, 0.f, 0.f), am_nxt = am_cur;
      if (h < GROUPS) {
        am_cur = load4(0);
        if (kchunks > 4) am_nxt = load4(4);
      }
      const bool pipelined = (u.nf4_regs & 6) == 6;
      uint4 p_next = make_uint4(0, 0, 0, 0);
      for (int c = 0; c < kchunks; ++c, ++nw, ++na) {
        const int s = nw % kSW, sa = na % kSA;
        if ((c & 3) == 0 && c > 0) {
          am_cur = am_nxt;
          if (h < GROUPS && c + 4 < kchunks) am_nxt = load4(c + 4);
        }
        const float a = (c & 3) == 0 ? am_cur.x : (c & 3) == 1 ? am_cur.y : (c & 3) == 2 ? am_cur.z : am_cur.w;
        // part p reads the row's 16-byte unit p (elements 32p .. 32p+31); with the pipelined decode
        // (flags 2 | 4) the next chunk's unit is loaded before this chunk's decode
        auto load_unit = [&](int slot) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (h < GROUPS) {
            const char* wsrc = smem + Smem::w + (slot * 2 + h) * kWBytes + r * 32;
            const int sw = (r >> 2) & 1;  // the 32-byte swizzle of the box (rows r and r + 4 apart)
            v = reinterpret_cast<const uint4*>(wsrc)[part ^ sw];
          }
          return v;
        };
        uint4 p0;
        if (pipelined && c > 0) {
          p0 = p_next;
        } else {
          if (!(tid == 128 ? STAT_WAIT(5, wt.wait(&full_w[s], (nw / kSW) & 1)) : wt.wait(&full_w[s], (nw / kSW) & 1))) break;
          p0 = load_unit(s);
        }
        if (pipelined && c + 1 < kchunks) {
          const int s1 = (nw + 1) % kSW;
          if (!wt.wait(&full_w[s1], ((nw + 1) / kSW) & 1)) break;
          p_next = load_unit(s1);
        }
        if (!(u.nf4_regs & 2)) {  // release the packed slot now (else after the decode, one fence for both)
          fence_proxy_async();  // generic reads of the slot before its refill by the async proxy
          mbar_arrive(&w_empty[s]);
        }
        if (!wt.wait(&a_empty[sa], ((na / kSA) & 1) ^ 1)) break;
#ifdef E4B_TRACE
        if (u.nf4_regs & 8) {  // trace builds only: skip the decode (timing of the other roles)
          fence_proxy_async();
          if (u.nf4_regs & 2) mbar_arrive(&w_empty[s]);
          mbar_arrive(&a_ready[sa]);
          continue;
        }
#endif
        if (h < GROUPS) {
          const uint32_t words[4] = {p0.x, p0.y, p0.z, p0.w};
          const __half2 sc = __float2half2_rn(a);
          char* adst = smem + Smem::a + (sa * 2 + h) * kABytes + r * 128;
          const int swz = (smem_u32(adst) >> 7) & 7;  // 128-byte swizzle follows the shared address
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {  // 16-byte unit q = 8 elements = packed word q
            const int q = 4 * part + qq;
            uint32_t o[4];
            if (u.nf4_regs & 1) {  // the same fp16 pairs from registers (byte permutes)
              uint32_t pr4[4];
              nf4_decode_word(words[qq], nfb, pr4);
#pragma unroll
              for (int bb = 0; bb < 4; ++bb) {
                __half2 v = __hmul2(*reinterpret_cast<__half2*>(&pr4[bb]), sc);
                o[bb] = *reinterpret_cast<uint32_t*>(&v);
              }
            } else
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
              const uint32_t byte = (words[qq] >> (8 * bb)) & 0xffu;
              uint32_t pr = *reinterpret_cast<const uint32_t*>(lut + ((byte << 7) | lane4));
              __half2 v = __hmul2(*reinterpret_cast<__half2*>(&pr), sc);
              o[bb] = *reinterpret_cast<uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(adst + ((q ^ swz) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        fence_proxy_async();
        if (u.nf4_regs & 2) mbar_arrive(&w_empty[s]);  // the packed bytes were consumed above
        mbar_arrive(&a_ready[sa]);
      }
      if (g.rank && !wt.dead) lora_chunk(ti, row);
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> global ---------------------------------
    // TMEM lane = token, column = feature: a thread owns one token row of the tile (the LoRA
    // delta is already in the accumulator: the MMA's extra K step). Gate column j and up column
    // 128 + j meet in one thread, and the row's 16-feature pieces leave as 16-byte stores.
    const int ew = warp - (4 + kDec / 32);  // TMEM lanes 32*ew .. 32*ew+31 (ew = warp % 4)
    const int r = ew * 32 + lane;      // token within the tile
    int it = 0;
    for (int t = unit0; t < total_tiles && !wt.dead; t += unit_step, ++it) {
      TileInfo ti;
      tile_info(s_ts, s_offs, g.E, nft, t, ti);
      const int buf = it & 1;
      float wsa = 1.f, wsb = 1.f;  // FP8: the tile's reference scales (gate rows, up rows)
      if (FMT == E4B_FMT_FP8_BLOCK128) {
        const int kbs = g.K / kFp8Block;
        const int rowA = group_row0(g, ti.ft, 0, GROUPS), rowB = group_row0(g, ti.ft, 1, GROUPS);
        const float* sa_ = g.absmax + ((int64_t)ti.e * (g.N / kFp8Block) + rowA / kFp8Block) * kbs;
        const float* sb_ = g.absmax + ((int64_t)ti.e * (g.N / kFp8Block) + rowB / kFp8Block) * kbs;
        float ma = 0.f, mb = 0.f;
        for (int kb = 0; kb < kbs; ++kb) {
          ma = fmaxf(ma, __ldg(sa_ + kb));
          if (GROUPS == 2) mb = fmaxf(mb, __ldg(sb_ + kb));
        }
        wsa = ma;
        wsb = mb;
      }
      const int m = PAIR ? ti.tt * 2 * kTok + (int)crank * kTok + r : ti.tt * kTok + r;
      const bool valid = m < ti.M;
      const int64_t srow = ti.row0 + (valid ? m : 0);
      float sc = 1.f;
      if (g.a_scale) sc = g.a_scale[g.a_rows ? g.a_rows[srow] : srow];
      if (PAIR) {  // warp-uniform wait: the warp later arrives once on the even CTA's acc_empty
        if (!__all_sync(0xffffffffu, wt.wait(&acc_full[buf], (it >> 1) & 1))) {
          wt.dead = true;
          break;
        }
      } else if (!(r == 0 ? STAT_WAIT(6, wt.wait(&acc_full[buf], (it >> 1) & 1)) : wt.wait(&acc_full[buf], (it >> 1) & 1))) {
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(ew * 32) << 16) + buf * 256;
      const bool swiglu = g.epilogue == E4B_EPI_SWIGLU;
      // SwiGLU: 128 outputs from gate (columns 0..127) and up (128..255); otherwise GROUPS x 128
      // consecutive outputs, column c -> feature ft * GROUPS * 128 + c
      const int halves = (GROUPS == 2 && !swiglu) ? 2 : 1;
      OutT* orow = reinterpret_cast<OutT*>(g.out) + srow * g.Nout + ti.ft * kRows * (swiglu ? 1 : GROUPS);
      for (int hh = 0; hh < halves; ++hh) {
        const float sh = sc * (hh == 0 ? wsa : wsb);
        for (int c0 = 0; c0 < kRows; c0 += 16) {
          float va[16], vb[16];
#ifdef E4B_TRACE
          long long tp0 = clock64();
#endif
          tmem_ld16(tbase + hh * kRows + c0, va);
          if (GROUPS == 2 && swiglu) tmem_ld16(tbase + kRows + c0, vb);
#ifdef E4B_TRACE
          long long tp1 = clock64();
          if (r == 0 && blockIdx.x < 148) atomicAdd(&g_umma_stats[blockIdx.x * 16 + 8], (unsigned long long)(tp1 - tp0));
#endif
          float o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float ya = va[i] * sh;
            if (GROUPS == 2 && swiglu)
              o[i] = silu_epi(ya) * (vb[i] * (sc * wsb));
            else if (g.epilogue == E4B_EPI_SILU)
              o[i] = silu_epi(ya);
            else
              o[i] = ya;
          }
          if (valid) {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const OutT lo = store_cast<OutT>(o[2 * j], g.err), hi = store_cast<OutT>(o[2 * j + 1], g.err);
              pk[j] = (uint32_t)(*reinterpret_cast<const uint16_t*>(&lo)) |
                      ((uint32_t)(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
#ifdef E4B_TRACE
            long long tp2 = clock64();
            if (r == 0 && blockIdx.x < 148) atomicAdd(&g_umma_stats[blockIdx.x * 16 + 9], (unsigned long long)(tp2 - tp1));
#endif
            uint4* dst = reinterpret_cast<uint4*>(orow + hh * kRows + c0);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
#ifdef E4B_TRACE
            if (r == 0 && blockIdx.x < 148) atomicAdd(&g_umma_stats[blockIdx.x * 16 + 10], (unsigned long long)(clock64() - tp2));
#endif
          }
        }
      }
      tc_fence_before();
      if (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(cluster_addr(&acc_empty[buf], 0));
      } else {
        mbar_arrive(&acc_empty[buf]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync_all();  // no CTA leaves while the other may still arrive on its barriers
  tc_fence_after();
  if (warp == 3) {
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
#ifdef E4B_TRACE
  if (tid == 0 && blockIdx.x < 148) atomicAdd(&g_umma_stats[blockIdx.x * 16 + 7], (unsigned long long)(clock64() - t_start));
#endif
}

size_t umma_workspace_bytes(int, int, int, int, int) { return 0; }

bool umma_eligible(int T, int k, int E, int H, int I, int has_gate, int act_dtype, int lora_rank) {
  (void)k;
  (void)E;
  (void)act_dtype;
  if (T <= 16) return false;  // the streaming GEMV owns decode shapes
  if (H % kKc || I % kKc) return false;
  // feature tiles of 128: gate_up produces I features (SwiGLU) or I (SiLU); down produces H
  if (I % kRows || H % kRows) return false;
  (void)has_gate;
  if (lora_rank > kEpiMaxRank || lora_rank % 4) return false;
  return encode_tiled_fn() != nullptr;
}

UmmaArgs umma_args_from(const GemvArgs& g, void* scratch, const int32_t* tile_start, int T, int k, int x_rows) {
  UmmaArgs u{};
  u.g = g;
  u.tile_start = tile_start;
  u.max_tiles = (T * k) / kUmmaTokens + (g.E < T * k ? g.E : T * k);
  u.x_rows = x_rows;
  u.scratch = scratch;
  return u;
}

template <typename OutT, int GROUPS, int FMT>
static e4b_status launch_groups(const UmmaArgs& u, cudaStream_t s) {
  using Smem = SmemT<FMT>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return E4B_ERR_CUDA;
  static unsigned long long configured = 0;
  static int sm_count[64] = {0};
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    if (cudaFuncSetAttribute(nf4_umma_kernel<OutT, GROUPS, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Smem::total) != cudaSuccess)
      return E4B_ERR_CUDA;
    cudaDeviceGetAttribute(&sm_count[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    configured |= bit;
  }
  const GemvArgs& g = u.g;
  const int nft = g.N / (GROUPS * kRows);
  int grid = sm_count[dev & 63];
  const int bound = u.max_tiles * nft;
  if (bound < grid) grid = bound;
  if (grid < 1) return E4B_OK;
  CUtensorMap wmap;  // weight bytes [E*N rows][K bytes per row (K/2 for NF4)], box {bytes of a chunk, 128 rows}
  const cuuint64_t row_bytes = FMT == E4B_FMT_FP8_BLOCK128 ? (cuuint64_t)g.K : (cuuint64_t)(g.K / 2);
  const cuuint64_t dims[2] = {row_bytes, (cuuint64_t)g.E * g.N};
  const cuuint64_t str[1] = {row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)Smem::wrow, kRows};
  // 32-byte rows (NF4, MXFP4) land with the 32-byte swizzle: a quarter-warp's 16-byte reads of rows
  // r .. r+7 then hit distinct banks; FP8's 64-byte rows are read in a rotated unit order instead
  const CUtensorMapSwizzle wsw = Smem::wrow == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (!encode_tiled(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, g.packed, dims, str, box, wsw))
    return E4B_ERR_CUDA;
  if (g.a_rows) return E4B_ERR_UNSUPPORTED;  // activations must be expert-sorted rows
  CUtensorMap bmap;  // fp16 activation rows [x_rows][K], box {64 halves, 128 rows}, 128-byte swizzle
  const cuuint64_t bdims[2] = {(cuuint64_t)g.K, (cuuint64_t)u.x_rows};
  const cuuint64_t bstr[1] = {(cuuint64_t)g.K * 2};
  const cuuint32_t bbox[2] = {kKc, kTok};
  const CUtensorMapDataType bdt = FMT == E4B_FMT_MXFP4 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (!encode_tiled(&bmap, bdt, 2, g.a, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B)) return E4B_ERR_CUDA;
  CUtensorMap lmap = bmap;  // LoRA-A products: fp16 rows of 64 (rank values, zero padded), same boxes
  if (g.rank) {
    if (!u.lora_xa16) return E4B_ERR_INVALID_ARG;
    const cuuint64_t ldims[2] = {64, (cuuint64_t)u.x_rows};
    const cuuint64_t lstr[1] = {128};
    if (!encode_tiled(&lmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, u.lora_xa16, ldims, lstr, bbox,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return E4B_ERR_CUDA;
  }
  // E4B_UMMA_FLAGS: bit 0 NF4 decode in registers; bit 1 a decode thread releases its packed-weight
  // slot after the chunk's decode, behind the one proxy fence that also publishes the decoded tile;
  // bit 2 (with bit 1) the decode loads the next chunk's packed units before decoding this one
  static const int nf4_regs = [] {
    const char* v = getenv("E4B_UMMA_FLAGS");
#ifdef E4B_TRACE
    return v ? atoi(v) & 127 : 6;
#else
    return v ? atoi(v) & 7 : 6;
#endif  // late release + pipelined decode by default (Qwen3 gate_up 477 -> 420 us)
  }();
  UmmaArgs ua = u;
  ua.nf4_regs = nf4_regs;
  if constexpr (FMT == E4B_FMT_NF4 && GROUPS == 2) {
    // E4B_UMMA_PAIR=1: clusters of two CTAs with tcgen05.mma.cta_group::2 (M = 256 tokens)
    static const bool pair = [] {
      const char* v = getenv("E4B_UMMA_PAIR");
      return v && atoi(v) != 0;
    }();
    if (pair) {
      auto kern = nf4_umma_kernel<OutT, GROUPS, FMT, true>;
      static int pair_clusters[64] = {0};
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.blockDim = dim3(kFwdThreads);
      cfg.dynamicSmemBytes = Smem::total;
      cfg.stream = s;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (!pair_clusters[dev & 63]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total) != cudaSuccess)
          return E4B_ERR_CUDA;
        cfg.gridDim = dim3(2 * (sm_count[dev & 63] / 2));
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) return E4B_ERR_CUDA;
        pair_clusters[dev & 63] = n;
      }
      int clusters = pair_clusters[dev & 63];
      if (bound < clusters) clusters = bound;  // token-pair tiles never outnumber the tiles
      cfg.gridDim = dim3(2 * clusters);
#ifdef E4B_TRACE
      fprintf(stderr, "[umma pair] clusters %d (max active %d), grid %d\n", clusters, pair_clusters[dev & 63], 2 * clusters);
#endif
      if (cudaLaunchKernelEx(&cfg, kern, ua, wmap, bmap, lmap) != cudaSuccess) return E4B_ERR_CUDA;
      return launch_status();
    }
  }
  nf4_umma_kernel<OutT, GROUPS, FMT><<<grid, kFwdThreads, Smem::total, s>>>(ua, wmap, bmap, lmap);
  return launch_status();
}

e4b_status launch_umma(const UmmaArgs& u, int act_dtype, cudaStream_t s, int weight_format) {
  (void)act_dtype;
  // two 128-row groups per tile: gate + up for SwiGLU, else 256 consecutive features when they divide N
  const bool two = u.g.epilogue == E4B_EPI_SWIGLU || u.g.N % (2 * kRows) == 0;
  if (weight_format == E4B_FMT_FP8_BLOCK128) {
    if (u.g.K % kFp8Block || u.g.N % kFp8Block || (u.g.epilogue == E4B_EPI_SWIGLU && (u.g.N / 2) % kFp8Block) ||
        u.g.rank)
      return E4B_ERR_UNSUPPORTED;
    if (u.g.out_dtype == E4B_BF16)
      return two ? launch_groups<__nv_bfloat16, 2, E4B_FMT_FP8_BLOCK128>(u, s)
                 : launch_groups<__nv_bfloat16, 1, E4B_FMT_FP8_BLOCK128>(u, s);
    return two ? launch_groups<__half, 2, E4B_FMT_FP8_BLOCK128>(u, s) : launch_groups<__half, 1, E4B_FMT_FP8_BLOCK128>(u, s);
  }
  if (weight_format == E4B_FMT_MXFP4) {  // bf16 operands and bf16 outputs (h, down rows)
    if (u.g.K % kKc || u.g.rank || u.g.out_dtype != E4B_BF16) return E4B_ERR_UNSUPPORTED;
    return two ? launch_groups<__nv_bfloat16, 2, E4B_FMT_MXFP4>(u, s)
               : launch_groups<__nv_bfloat16, 1, E4B_FMT_MXFP4>(u, s);
  }
  if (u.g.out_dtype == E4B_BF16)
    return two ? launch_groups<__nv_bfloat16, 2, E4B_FMT_NF4>(u, s) : launch_groups<__nv_bfloat16, 1, E4B_FMT_NF4>(u, s);
  return two ? launch_groups<__half, 2, E4B_FMT_NF4>(u, s) : launch_groups<__half, 1, E4B_FMT_NF4>(u, s);
}

// ---------------------------------------------------------------------------------------------
// dgrad: dX[r, :] = dY[r, :] . W_e for the expert-sorted rows r of expert e (W_e [N, K] NF4,
// blocks of 64 along K): the input gradient of a frozen grouped projection, the reference's
// single-launch dgrad kernel (experts4bit_qlora/engines/fast.py:519-550) without materialising
// a decoded stack. The contraction runs over N (the weight rows): per 64-row chunk the decode
// warps turn 64 rows x 256 columns of the tile into fp16 and store each row's 64-column pieces
// as 128-byte rows of MN-major, 128-byte-swizzled atoms (8 weight rows x 64 columns), which the
// MMA reads as its N = 256 operand with the MN-major bit set (LBO: the next 64 columns, SBO: the
// next 8 rows). The M = 128 operand is the tile's fp16 dY rows (per-row power-of-two scales,
// multiplied back in the epilogue), K-major over N like the forward activations. Same roles and
// rings as the forward kernel; the epilogue stores fp32 or 16-bit rows of 256 columns.
namespace {

// MN-major, 128-byte swizzle descriptor: atoms of 8 K-rows x 128 B, `lbo` bytes to the next atom
// along MN, `sbo` bytes to the next 8 K-rows.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fff);
  d |= (uint64_t)((lbo >> 4) & 0x3fff) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fff) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

constexpr int kDgCols = 256;  // output columns (of K) per tile
constexpr int kDgAtom = 1024;

}  // namespace

template <typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_umma_dgrad_kernel(UmmaArgs u, const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap bmap) {
  using Smem = SmemT<E4B_FMT_NF4>;
  static_assert(Smem::wbytes * 2 == 64 * 128, "one packed stage holds 64 rows x 128 bytes");
  static_assert(2 * kABytes == kDgCols * 64 * 2, "one decoded stage holds 64 rows x 256 columns");
  extern __shared__ __align__(1024) char smem[];
  const GemvArgs& g = u.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  char* lut = smem + Smem::lut;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::bars);
  uint64_t* full_w = bars;
  uint64_t* w_empty = full_w + kSW;
  uint64_t* full_b = w_empty + kSW;
  uint64_t* b_empty = full_b + kSB;
  uint64_t* a_ready = b_empty + kSB;
  uint64_t* a_empty = a_ready + kSA;
  uint64_t* acc_full = a_empty + kSA;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Smem::tmem_slot);
  int32_t* s_ts = reinterpret_cast<int32_t*>(smem + Smem::tables);
  int32_t* s_offs = s_ts + 1025;
  for (int i = tid; i <= g.E; i += kThreads) {
    s_ts[i] = u.tile_start[i];
    s_offs[i] = g.offsets[i];
  }
  const int nct = g.K / kDgCols;  // column tiles per expert
  const int nchunks = g.N / 64;   // 64 weight rows per chunk
  const int total_tiles = u.tile_start[g.E] * nct;
  Waiter wt{false, g.err};
  if (tid == 0) {
    for (int s = 0; s < kSW; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&w_empty[s], 256);
    }
    for (int s = 0; s < kSB; ++s) {
      mbar_init(&full_b[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kSA; ++s) {
      mbar_init(&a_ready[s], 256);
      mbar_init(&a_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    fence_proxy_async();
  }
  if (warp == 3) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  {
    const float code = c_nf4[lane & 15];
    for (int e = warp; e < 256; e += kThreads / 32) {
      const float lo = __shfl_sync(0xffffffffu, code, e >> 4), hi = __shfl_sync(0xffffffffu, code, e & 15);
      reinterpret_cast<uint32_t*>(lut)[e * 32 + lane] = pack2<__half>(lo, hi);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // packed rows: one box {128 B = 256 columns, 64 rows} per chunk, 128-byte swizzle
    if (lane == 0) {
      int n = 0;
      for (int t = blockIdx.x; t < total_tiles && !wt.dead; t += gridDim.x) {
        TileInfo ti;
        tile_info(s_ts, s_offs, g.E, nct, t, ti);
        for (int c = 0; c < nchunks; ++c, ++n) {
          const int s = n % kSW;
          if (!wt.wait(&w_empty[s], ((n / kSW) & 1) ^ 1)) break;
          mbar_arrive_expect_tx(&full_w[s], 64 * 128);
          tma_load_2d(smem + Smem::w + s * 2 * Smem::wbytes, &wmap, ti.ft * (kDgCols / 2), ti.e * g.N + c * 64,
                      &full_w[s]);
        }
      }
    }
  } else if (warp == 1) {
    // dY rows: one box {64 columns of N, 128 rows} per chunk
    if (lane == 0) {
      int n = 0;
      for (int t = blockIdx.x; t < total_tiles && !wt.dead; t += gridDim.x) {
        TileInfo ti;
        tile_info(s_ts, s_offs, g.E, nct, t, ti);
        for (int c = 0; c < nchunks; ++c, ++n) {
          const int s = n % kSB;
          if (!wt.wait(&b_empty[s], ((n / kSB) & 1) ^ 1)) break;
          mbar_arrive_expect_tx(&full_b[s], kBBytes);
          tma_load_2d(smem + Smem::b + s * kBBytes, &bmap, c * 64, ti.row0 + ti.tt * kTok, &full_b[s]);
        }
      }
    }
  } else if (warp == 2) {
    // idle
  } else if (warp == 3) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kDgCols) | (1u << 16);  // B (the decoded weights) MN-major
      int n = 0, it = 0;
      for (int t = blockIdx.x; t < total_tiles && !wt.dead; t += gridDim.x, ++it) {
        const int buf = it & 1;
        if (!wt.wait(&acc_empty[buf], ((it >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        for (int c = 0; c < nchunks; ++c, ++n) {
          const int s = n % kSB, sa = n % kSA;
          if (!wt.wait(&full_b[s], (n / kSB) & 1)) break;
          if (!wt.wait(&a_ready[sa], (n / kSA) & 1)) break;
          tc_fence_after();
          const uint32_t ysm = smem_u32(smem + Smem::b + s * kBBytes);
          const uint32_t wsm = smem_u32(smem + Smem::a + sa * 2 * kABytes);
          for (int kk = 0; kk < 4; ++kk)  // 16 weight rows = two 8-row atoms per step
            umma_f16(tmem + buf * kDgCols, sw128_desc(ysm + kk * 32),
                     sw128_mn_desc(wsm + kk * 2 * kDgAtom, 8 * kDgAtom, kDgAtom), idesc, (c | kk) != 0);
          umma_commit(&b_empty[s]);
          umma_commit(&a_empty[sa]);
        }
        umma_commit(&acc_full[buf]);
      }
    }
  } else if (warp < 12) {
    // decode: thread (row rr of the chunk, column atom kb) turns 32 packed bytes into 64 fp16
    const int d = tid - 128;
    const int rr = d & 63, kb = d >> 6;
    const uint32_t lane4 = (uint32_t)lane << 2;
    int nw = 0;
    for (int t = blockIdx.x; t < total_tiles && !wt.dead; t += gridDim.x) {
      TileInfo ti;
      tile_info(s_ts, s_offs, g.E, nct, t, ti);
      const float* am = g.absmax + ((int64_t)ti.e * g.N + rr) * (g.K / 64) + ti.ft * 4 + kb;
      float a_nxt = __ldg(am);
      for (int c = 0; c < nchunks; ++c, ++nw) {
        const int s = nw % kSW, sa = nw % kSA;
        const float a = a_nxt;
        if (c + 1 < nchunks) a_nxt = __ldg(am + (int64_t)(c + 1) * 64 * (g.K / 64));
        if (!wt.wait(&full_w[s], (nw / kSW) & 1)) break;
        const char* wrow = smem + Smem::w + s * 2 * Smem::wbytes + rr * 128;
        const uint4 p0 = *reinterpret_cast<const uint4*>(wrow + (((2 * kb) ^ (rr & 7)) << 4));
        const uint4 p1 = *reinterpret_cast<const uint4*>(wrow + (((2 * kb + 1) ^ (rr & 7)) << 4));
        if (!wt.wait(&a_empty[sa], ((nw / kSA) & 1) ^ 1)) break;
        const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const __half2 sc = __float2half2_rn(a);
        char* adst = smem + Smem::a + sa * 2 * kABytes + (kb * 8 + (rr >> 3)) * kDgAtom + (rr & 7) * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // 16-byte unit q = columns 8q .. 8q+7 of the atom
          uint32_t o[4];
#pragma unroll
          for (int bb = 0; bb < 4; ++bb) {
            const uint32_t byte = (words[q] >> (8 * bb)) & 0xffu;
            uint32_t pr = *reinterpret_cast<const uint32_t*>(lut + ((byte << 7) | lane4));
            __half2 v = __hmul2(*reinterpret_cast<__half2*>(&pr), sc);
            o[bb] = *reinterpret_cast<uint32_t*>(&v);
          }
          *reinterpret_cast<uint4*>(adst + ((q ^ (rr & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        // one proxy fence orders the packed-slot reads (consumed above) before its refill and the
        // decoded tile's writes before the MMA's reads
        fence_proxy_async();
        mbar_arrive(&w_empty[s]);
        mbar_arrive(&a_ready[sa]);
      }
    }
  } else {
    // epilogue: TMEM lane = row of the token tile, column = output column of the tile
    const int ew = warp - 12;
    const int r = ew * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < total_tiles && !wt.dead; t += gridDim.x, ++it) {
      TileInfo ti;
      tile_info(s_ts, s_offs, g.E, nct, t, ti);
      const int buf = it & 1;
      const int m = ti.tt * kTok + r;
      const bool valid = m < ti.M;
      const int64_t srow = ti.row0 + (valid ? m : 0);
      const float sc = g.a_scale ? g.a_scale[srow] : 1.f;
      if (!wt.wait(&acc_full[buf], (it >> 1) & 1)) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(ew * 32) << 16) + buf * kDgCols;
      OutT* orow = reinterpret_cast<OutT*>(g.out) + srow * g.Nout + ti.ft * kDgCols;
      for (int c0 = 0; c0 < kDgCols; c0 += 16) {
        float v[16];
        tmem_ld16(tbase + c0, v);
        if (valid) {
          if (sizeof(OutT) == 4) {
            float4* dst = reinterpret_cast<float4*>(orow + c0);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_float4(v[4 * j] * sc, v[4 * j + 1] * sc, v[4 * j + 2] * sc, v[4 * j + 3] * sc);
          } else {
            uint32_t pk[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const OutT lo = store_cast<OutT>(v[2 * j] * sc, g.err), hi = store_cast<OutT>(v[2 * j + 1] * sc, g.err);
              pk[j] = (uint32_t)(*reinterpret_cast<const uint16_t*>(&lo)) |
                      ((uint32_t)(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(orow + c0);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 3) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

bool umma_dgrad_eligible(int N, int K) { return N % 64 == 0 && K % kDgCols == 0 && encode_tiled_fn() != nullptr; }

template <typename OutT>
static e4b_status launch_dgrad_t(const UmmaArgs& u, cudaStream_t s) {
  using Smem = SmemT<E4B_FMT_NF4>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return E4B_ERR_CUDA;
  static std::atomic<unsigned long long> configured{0};
  static int sm_count[64] = {0};
  const unsigned long long bit = 1ull << dev;
  if (!(configured.load() & bit)) {
    if (cudaFuncSetAttribute(nf4_umma_dgrad_kernel<OutT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total) !=
        cudaSuccess)
      return E4B_ERR_CUDA;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sm_count[dev] = sms;
    configured.fetch_or(bit);
  }
  const GemvArgs& g = u.g;
  int grid = sm_count[dev];
  const int bound = u.max_tiles * (g.K / kDgCols);
  if (bound < grid) grid = bound;
  if (grid < 1) return E4B_OK;
  CUtensorMap wmap;  // packed rows [E*N][K/2 bytes], box {128 B, 64 rows}, 128-byte swizzle
  const cuuint64_t dims[2] = {(cuuint64_t)(g.K / 2), (cuuint64_t)g.E * g.N};
  const cuuint64_t str[1] = {(cuuint64_t)(g.K / 2)};
  const cuuint32_t box[2] = {128, 64};
  if (!encode_tiled(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, g.packed, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B))
    return E4B_ERR_CUDA;
  CUtensorMap bmap;  // fp16 dY rows [x_rows][N], box {64, 128 rows}, 128-byte swizzle
  const cuuint64_t bdims[2] = {(cuuint64_t)g.N, (cuuint64_t)u.x_rows};
  const cuuint64_t bstr[1] = {(cuuint64_t)g.N * 2};
  const cuuint32_t bbox[2] = {64, kTok};
  if (!encode_tiled(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, g.a, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B))
    return E4B_ERR_CUDA;
  nf4_umma_dgrad_kernel<OutT><<<grid, kThreads, Smem::total, s>>>(u, wmap, bmap);
  return launch_status();
}

e4b_status launch_umma_dgrad(const UmmaArgs& u, int out_dtype, cudaStream_t s) {
  if (!umma_dgrad_eligible(u.g.N, u.g.K)) return E4B_ERR_UNSUPPORTED;
  switch (out_dtype) {
    case E4B_F32: return launch_dgrad_t<float>(u, s);
    case E4B_BF16: return launch_dgrad_t<__nv_bfloat16>(u, s);
    case E4B_F16: return launch_dgrad_t<__half>(u, s);
    default: return E4B_ERR_UNSUPPORTED;
  }
}

}  // namespace e4b
