// Internal launch interface of the tcgen05 grouped NF4 GEMM (prefill regime).
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace e4b {

constexpr int kUmmaTokens = 128;   // token tile (UMMA N) per CTA

struct UmmaArgs {
  GemvArgs g;                      // operands, epilogue and LoRA, as for the GEMV
  const int32_t* tile_start;       // [E+1] prefix of ceil(count / kUmmaTokens)
  int max_tiles;
  int x_rows;                      // rows of the activation matrix g.a
  void* scratch;
  const __half* lora_xa16;         // [x_rows, 64] fp16: scaling * (x16_row . A^T), zero padded (rank > 0)
  int nf4_regs;                    // bit 0: NF4 decode by register byte permutes; bit 1: late slot release
};

// Rows per expert (on average) from which the tensor-core path beats the GEMV, which
// re-reads an expert's weights for every 16 of its rows.
constexpr int kUmmaMinRowsPerExpert = 16;
inline bool umma_worthwhile(int64_t rows, int experts) { return rows >= (int64_t)kUmmaMinRowsPerExpert * experts; }

size_t umma_workspace_bytes(int T, int k, int E, int H, int I);
bool umma_eligible(int T, int k, int E, int H, int I, int has_gate, int act_dtype, int lora_rank);
UmmaArgs umma_args_from(const GemvArgs& g, void* scratch, const int32_t* tile_start, int T, int k, int x_rows);
e4b_status launch_umma(const UmmaArgs& u, int act_dtype, cudaStream_t s, int weight_format = E4B_FMT_NF4);

// dgrad of a frozen grouped NF4 projection (umma.cu): out[r, :K] = a[r, :N] . W_e with `a` fp16
// expert-sorted rows [x_rows, N] (per-row scales in g.a_scale), out_dtype fp32 / bf16 / fp16,
// g.Nout = K. N a multiple of 64, K of 256; tile_start counts kUmmaTokens-row tiles.
bool umma_dgrad_eligible(int N, int K);
e4b_status launch_umma_dgrad(const UmmaArgs& u, int out_dtype, cudaStream_t s);

}  // namespace e4b
