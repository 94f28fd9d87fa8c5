// Internal launch interface of the LoRA-A pre-pass.
#pragma once
#include "common.cuh"

namespace e4b {

struct LoraAArgs {
  const __half* a;           // activations, fp16 rows of K
  const float* a_scale;      // nullable: per source row power-of-two scale of `a`
  const int32_t* a_rows;     // nullable gather map (sorted row -> source row)
  const void* loraA;         // [E, rank, K] (lora dtype)
  const int32_t* offsets;    // [E+1]
  const int32_t* tile_start; // [E+1] prefix of ceil(count / kLoraRows)
  int E, K, rank, lora_dtype;
  float scaling;
  float* xa;                 // [R, rank] fp32 = scaling * (a_row . A[e]^T) (a_scale applied)
  __half* xa16;              // instead of xa when set: [R, 64] fp16 = scaling * (a_row . A[e]^T) without
                             // a_scale, ranks zero padded to 16 (the tensor-core GEMM's extra K step)
  int max_tiles;
};
constexpr int kLoraRows = 64;
constexpr int kLoraMaxRank = 64;

e4b_status launch_lora_a(const LoraAArgs& g, cudaStream_t s);

}  // namespace e4b
