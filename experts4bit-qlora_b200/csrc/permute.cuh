// Internal launch interface of the permutation kernel (shared with moe.cu).
#pragma once
#include "common.cuh"
#include "convert.cuh"

namespace e4b {

struct PermuteArgs {
  const int64_t* topk_idx;  // [T*k]
  int T, k, E;
  const int32_t* emap;      // optional routed id -> stack index (see stack_expert)
  int routed;               // routed ids with a map
  int32_t* order;           // [T*k] sorted row -> flat index (nullable)
  int32_t* inv;             // [T*k] flat index -> sorted row (nullable)
  int32_t* sorted_token;    // [T*k] sorted row -> token (nullable)
  int32_t* offsets;         // [E+1]
  int32_t* active;          // [E] active expert ids, ascending (nullable)
  int32_t* num_active;      // [1] (nullable)
  int32_t* tile_start_a;    // [E+1] prefix of ceil(count/tile_a) (nullable)
  int32_t* tile_start_b;    // [E+1] prefix of ceil(count/tile_b) (nullable)
  int tile_a, tile_b;
  int* err;                 // device error word
  int reset_err;            // zero *err before validating (first kernel of a call)
  ConvertArgs conv;         // optional: rows converted to fp16 by CTAs 1.. of the same launch
  int conv_ctas;
  int32_t* seg_scratch;     // optional: permute_scratch_bytes(T*k, E) of global memory; with it,
                            // large inputs take the multi-CTA permutation (same result)
};

size_t permute_smem_bytes(int E);
// Global scratch of the multi-CTA permutation (0 below its size threshold).
size_t permute_scratch_bytes(int64_t n, int E);
e4b_status launch_permute(const PermuteArgs& a, cudaStream_t s);

}  // namespace e4b
