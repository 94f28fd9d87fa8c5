// Internal interface of the one-launch decode layer kernel (decode_layer.cu).
#pragma once
#include "common.cuh"

namespace e4b {

// Whether the fused decode-layer kernel takes this layer (NF4, <= 128 picks, no
// adapters, H and I multiples of 256, token rows within 20 KB of shared memory).
bool decode_layer_eligible(const e4b_moe_desc& d);
// Workspace bytes of its per-CTA error slots.
size_t decode_layer_sync_bytes(int grid);
// h [R, I] and down_rows [R, H] are fp16 scratch; `sync` holds
// decode_layer_sync_bytes(grid) bytes (rewritten by every launch).
// Optional router fused in front of the layer (instead of the two router kernels): every CTA
// computes the T x E logits of x . W_r^T (T * E <= 4096) and the top-k, written to
// topk_idx / topk_w [T, k] by CTA 0.
struct DecodeRouter {
  const void* weight;
  int weight_dtype, kind, norm_topk_prob;
  int64_t* topk_idx;
  float* topk_w;
  float* logits;  // [T, E] fp32 scratch in global memory: logits computed across the grid (null: per CTA)
};
bool decode_router_fusable(const e4b_moe_desc& d);

// 0 off, 1 flow kernel where it applies (else the phase kernel), 2 phase kernel only, 3 slice
// kernel where it applies (else the phase kernel).
int decode_mode();
// Shapes the slice kernel takes (gated NF4 layer, 1..8 tokens, H a multiple of 512, within the
// phase kernel's limits), and the bytes of its fp32 partial down rows [T*k][I / 64][H].
bool decode_slice_shape(const e4b_moe_desc& d);
size_t decode_slice_part_bytes(const e4b_moe_desc& d);

// The flow kernel (decode_flow.cu): the layer for 1..8 tokens and at most kFlowMaxPicks picks,
// NF4, no adapters, H and I multiples of 256. `sync` is the workspace's counter block at
// kFlowSyncOffset ((kFlowMaxPicks + 1) words, zero before the first launch, left zero by every
// launch); h is [T*k, I] fp16 scratch. With `router`, the router runs inside the launch (its
// logits never leave the thread-block cluster) and writes topk_idx / topk_w.
constexpr int kFlowMaxPicks = 64;
bool decode_flow_eligible(const e4b_moe_desc& d, bool fused_router);
e4b_status launch_decode_flow(const e4b_moe_desc& d, const e4b_moe_tensors* t, void* h, void* sync, int* err,
                              cudaStream_t s, const DecodeRouter* router = nullptr);
// `part` (decode_slice_part_bytes) enables the slice kernel in mode 3; null keeps the phase kernel.
e4b_status launch_decode_layer(const e4b_moe_desc& d, const e4b_moe_tensors* t, void* h, void* down_rows,
                               void* sync, int* err, cudaStream_t s, const DecodeRouter* router = nullptr,
                               void* part = nullptr);

}  // namespace e4b
