// NF4 decode without shared memory: the codebook's fp16 bytes in registers and byte permutes
// (prmt) that turn a packed word into the four fp16 pairs the pair table would return. Used where
// the shared-memory pipe, not the integer pipe, is the contended resource.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "common.cuh"

namespace e4b {

// The NF4 codebook as fp16 bytes in registers, for the byte-permute decode: l0..l3 hold the low
// bytes of codes 0-3, 4-7, 8-11, 12-15 and h0..h3 the high bytes.
struct Nf4Bytes {
  uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
};

__device__ __forceinline__ Nf4Bytes nf4_bytes() {
  uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
#pragma unroll
  for (int v = 0; v < 16; ++v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(c_nf4[v]));
    lo[v >> 2] |= (b & 0xffu) << (8 * (v & 3));
    hi[v >> 2] |= (b >> 8) << (8 * (v & 3));
  }
  return Nf4Bytes{lo[0], lo[1], lo[2], lo[3], hi[0], hi[1], hi[2], hi[3]};
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
  return d;
}
__device__ __forceinline__ uint32_t bytesel(uint32_t a, uint32_t b, uint32_t m) {  // (a & ~m) | (b & m)
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(d) : "r"(a), "r"(b), "r"(m));
  return d;
}

// The four fp16 pairs of a packed word (byte j -> the pair table's entry j: code[high nibble] in
// the low half) with no shared memory: a 3-bit index selects a byte of an 8-entry half of the
// table (prmt), bit 3 of each nibble (spread to a byte mask by prmt's sign replication) picks
// the half. Bit-identical to the pair-table lookups.
__device__ __forceinline__ void nf4_decode_word(uint32_t w, const Nf4Bytes& T, uint32_t (&o)[4]) {
  const uint32_t t = w << 4;
  const uint32_t s = w & 0x77777777u, sh = s >> 16;
  const uint32_t m0 = prmt(t, w, 0xD9C8u), m1 = prmt(t, w, 0xFBEAu);
  const uint32_t la = bytesel(prmt(T.l0, T.l1, s), prmt(T.l2, T.l3, s), m0);
  const uint32_t ha = bytesel(prmt(T.h0, T.h1, s), prmt(T.h2, T.h3, s), m0);
  const uint32_t lb = bytesel(prmt(T.l0, T.l1, sh), prmt(T.l2, T.l3, sh), m1);
  const uint32_t hb = bytesel(prmt(T.h0, T.h1, sh), prmt(T.h2, T.h3, sh), m1);
  o[0] = prmt(la, ha, 0x4051u);
  o[1] = prmt(la, ha, 0x6273u);
  o[2] = prmt(lb, hb, 0x4051u);
  o[3] = prmt(lb, hb, 0x6273u);
}

}  // namespace e4b
