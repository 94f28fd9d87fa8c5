// tcgen05 grouped NF4 GEMM for the prefill regime.
#include "umma.cuh"

namespace e4b {

size_t umma_workspace_bytes(int, int, int, int, int) { return 0; }

bool umma_eligible(int, int, int, int, int, int, int) { return false; }

UmmaArgs umma_args_from(const GemvArgs& g, void* scratch, const int32_t* tile_start, int T, int k) {
  UmmaArgs u{};
  u.g = g;
  u.tile_start = tile_start;
  u.max_tiles = (T * k) / kUmmaTokens + (g.E < T * k ? g.E : T * k);
  u.scratch = scratch;
  return u;
}

e4b_status launch_umma(const UmmaArgs&, int, cudaStream_t) { return E4B_ERR_UNSUPPORTED; }

}  // namespace e4b
