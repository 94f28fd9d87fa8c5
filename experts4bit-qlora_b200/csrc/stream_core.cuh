// Building blocks of the streaming NF4 GEMV (gemv_stream.cu) shared with the
// decode-layer kernel (decode_layer.cu): ring geometry, the pair-table address
// math, the fragment offsets inside a swizzled TMA box, and the tile helpers.
#pragma once
#include "async.cuh"
#include "gemv.cuh"

namespace e4b {
namespace stream {

constexpr int kPairs = 8;                   // warp pairs per CTA
constexpr int kWarps = 2 * kPairs;
constexpr int kThreads = kWarps * 32;
constexpr int kSlots = 3;
constexpr int kChunk = 512;                 // K elements per chunk = 2 lines of 128 B per row
constexpr int kBoxW = 8 * 2 * 128;          // one 8-row group of packed bytes
constexpr int kBoxA = 8 * 8 * 4;            // one 8-row group of absmax (8 blocks)
constexpr int kSlotBytes = 5120;            // 2 x kBoxW + 2 x kBoxA, padded to keep 1024-B alignment
constexpr uint32_t kItemTx = 2 * kBoxW + 2 * kBoxA;
constexpr int kLut = 256 * 128;             // 32 KB pair table
constexpr int kXBudget = 64 * 1024;         // activation rows staged per CTA
constexpr int kXRegs = kXBudget / 16 / kThreads;  // 16-byte activation vectors per thread

struct Smem {
  static constexpr int lut = 0;
  static constexpr int x = kLut;
  static constexpr int slots = kLut + kXBudget;  // 96 KB: 1024-aligned for the swizzled boxes
  static constexpr int red = slots + kPairs * kSlots * kSlotBytes;
  static constexpr int bars = red + kPairs * 32 * 8 * 4;
  static constexpr int total = bars + kPairs * kSlots * 8;
};

// Table entry address of byte POS of `word` for this lane: ((byte << 7) | lane4).
template <int POS>
__device__ __forceinline__ uint32_t lut_addr(uint32_t word, uint32_t lane4) {
  const uint32_t sh = POS == 0 ? (word << 7) : (word >> (8 * POS - 7));
  uint32_t a;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(a) : "r"(sh), "r"(0x7F80u), "r"(lane4));  // (sh & m) | lane4
  return a;
}
template <int POS>
__device__ __forceinline__ uint32_t lut2(const char* lut, uint32_t word, uint32_t lane4) {
  return *reinterpret_cast<const uint32_t*>(lut + lut_addr<POS>(word, lane4));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

struct Tile {
  int e, row0, M, tile;
};

__device__ __forceinline__ void tile_of(const GemvArgs& g, int t, Tile& out) {
  const int j = t / g.tiles_per_expert;
  out.tile = t - j * g.tiles_per_expert;
  out.e = g.active[j];
  out.row0 = g.offsets[out.e];
  out.M = g.offsets[out.e + 1] - out.row0;
}

// First weight row of 8-row group h (0: MMA rows 0-7, 1: MMA rows 8-15) of a tile.
__device__ __forceinline__ int group_row(const GemvArgs& g, int tile, int h) {
  if (g.epilogue == E4B_EPI_SWIGLU) return h == 0 ? tile * 8 : (g.N >> 1) + tile * 8;
  return tile * 16 + 8 * h;
}

// Byte offset of lane (row r of the group, quad lane q) 8-byte piece of block b in a
// 128-byte-swizzled box whose shared address is `box`. The swizzle XORs the 16-byte
// unit index with bits 7-9 of the shared address, so it is computed from the address.
__device__ __forceinline__ int wofs(uint32_t box, int r, int q, int b) {
  const int line = 2 * r + (b >> 2);  // a 128-byte line holds four 32-byte blocks
  const int unit = (((b & 3) << 1) | (q >> 1)) ^ (((box >> 7) + line) & 7);
  return line * 128 + (unit << 4) + ((q & 1) << 3);
}

}  // namespace stream
}  // namespace e4b
