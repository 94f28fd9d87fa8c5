// Internal launch interface of the grouped NF4 GEMV (decode regime).
#pragma once
#include "common.cuh"

namespace e4b {

struct GemvArgs {
  const void* a;             // activations, rows of K elements, fp16 (see convert.cuh)
  const float* a_scale;      // nullable: per source row power-of-two scale of `a`
  const int32_t* a_rows;     // nullable: sorted row r reads a[a_rows[r]]
  const uint8_t* packed;     // [E, N, K/2]
  const float* absmax;       // [E, N, K/64]
  const int32_t* offsets;    // [E+1] sorted-row start of each expert
  const int32_t* active;     // [E] active expert ids (ascending)
  const int32_t* num_active; // [1]
  int E, N, K;
  int epilogue;              // e4b_epilogue
  void* out;                 // [R, Nout] out_dtype (bf16 or fp16; fp16 saturates and flags)
  int out_dtype;
  int Nout;
  const float* lora_xa;      // [R, rank] = scaling * (a_row . A^T), fp32 (nullable)
  const void* lora_B;        // [E, N, rank] (lora_dtype)
  int lora_dtype, rank;
  int tiles_per_expert;      // MMA row tiles per expert
  int max_tasks;             // upper bound on tasks (max active experts x tiles)
  int* err;
};

// Tokens per expert handled without re-reading the weights.
constexpr int kGemvMaxCols = 16;

e4b_status launch_gemv(const GemvArgs& g, int max_rows_per_expert, cudaStream_t s);

// Streaming variant (gemv_stream.cu): activation rows [x_rows, K] staged in
// shared memory, weights streamed by per-warp bulk-copy rings.
bool gemv_stream_eligible(const GemvArgs& g, int x_rows, int max_rows_per_expert);
e4b_status launch_gemv_stream(const GemvArgs& g, int x_rows, int max_rows_per_expert, cudaStream_t s);

// Block-scaled FP8 weights (fp8.cu): bf16 activations, `absmax` holds the fp32 tile scales.
e4b_status launch_fp8_gemv(const GemvArgs& g, cudaStream_t s);

// Picks the streaming kernel when eligible, else the general one.
inline e4b_status launch_gemv_auto(const GemvArgs& g, int x_rows, int max_rows_per_expert, cudaStream_t s) {
  if (gemv_stream_eligible(g, x_rows, max_rows_per_expert)) return launch_gemv_stream(g, x_rows, max_rows_per_expert, s);
  return launch_gemv(g, max_rows_per_expert, s);
}

}  // namespace e4b
