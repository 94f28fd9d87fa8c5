// Internal interface of the expert stages of a layer (shared by the fused layer
// in moe.cu and the expert-parallel expert side in ep.cu).
#pragma once
#include "common.cuh"
#include "convert.cuh"

namespace e4b {

// Rows already grouped by expert, with their segment tables, and the scratch the
// stages write. `x16` holds fp16 activations with per-row power-of-two scales.
struct ExpertRows {
  const __half* x16;            // fp16 rows with per-row power-of-two scales
  const float* x_scale;
  const int32_t* a_rows;        // nullable: sorted row r reads x16[a_rows[r]] (streaming path only)
  int x_rows;                   // rows of x16
  int R;                        // sorted rows
  int max_rows_per_expert;      // upper bound on any expert's segment
  const int32_t* offsets;       // [E+1]
  const int32_t* active;        // [E] ascending
  const int32_t* num_active;    // [1]
  const int32_t* tile_a;        // [E+1] prefix of ceil(count / kLoraRows)
  const int32_t* tile_b;        // [E+1] prefix of ceil(count / kUmmaTokens)
  bool use_umma;                // tensor-core GEMM (x16 expert-sorted, a_rows null)
  void* h;                      // [R, I] fp16
  void* down_rows;              // [R, H] fp16, unweighted, sorted order
  float* xa_gu;                 // [R, rank] (LoRA only)
  float* xa_dn;
  void* umma_scratch;
  int* err;
};

// Records stage event i of t->stage_events (if any) on s, as an external graph
// node while s is capturing.
void mark_stage(const e4b_moe_tensors* t, int i, cudaStream_t s);

// [LoRA-A of x] -> gate_up GEMM (+LoRA, SwiGLU) -> [LoRA-A of h] -> down GEMM (+LoRA).
// Marks stages 1..5. Weights and adapters come from t; d.num_experts is the number
// of experts those stacks hold.
e4b_status run_expert_stages(const e4b_moe_desc& d, const e4b_moe_tensors* t, const ExpertRows& x, cudaStream_t s);

// Grid size for the row-conversion kernels (8 or 32 warps per CTA).
int conv_ctas_for(int rows, int warps_per_cta);
// dst[r] = fp16(src[rows_map[r]]) with per-row power-of-two scales (convert.cuh).
e4b_status launch_gather_convert(const ConvertArgs& c, const int32_t* rows_map, cudaStream_t s);
// dst[r] = src[rows_map[r]] for rows of K 16-bit elements (K % 8 == 0), no conversion.
e4b_status launch_gather_rows16(const void* src, const int32_t* rows_map, int rows, int K, void* dst, cudaStream_t s);
// Validation shared by the fused layer entry points.
e4b_status check_weight_format(const e4b_moe_desc& d);

}  // namespace e4b
