// Whole expert layer and the standalone grouped GEMM entry point.
//
// e4b_moe_forward is the device-side replacement of fused_experts_forward /
// fused_experts_lora_forward (experts4bit_qlora/engines/fast.py:100-257):
//   permute (no host sync) -> [LoRA-A of x] -> grouped gate_up GEMM with the
//   LoRA delta and SwiGLU fused -> [LoRA-A of h] -> grouped down GEMM with its
//   LoRA delta -> weighted fixed-order combine.
// All launches are stream-ordered on the caller's stream; nothing is allocated.
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "convert.cuh"
#include "gemv.cuh"
#include "lora.cuh"
#include "permute.cuh"
#include "umma.cuh"
#include "moe_stages.cuh"
#include "decode_layer.cuh"

namespace e4b {

struct MoeLayout {
  size_t offsets, active, num_active, tile_a, tile_b, inv, sorted_token, x16, x_scale, h, down_rows, xa_gu, xa_dn,
      umma, sync, part, perm, total;
};

static MoeLayout moe_layout(const e4b_moe_desc& d) {
  MoeLayout L{};
  const size_t R = (size_t)d.tokens * d.top_k;
  const size_t E = d.num_experts;
  size_t o = kErrBytes;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  L.offsets = take((E + 1) * 4);
  L.active = take(E * 4);
  L.num_active = take(4);
  L.tile_a = take((E + 1) * 4);
  L.tile_b = take((E + 1) * 4);
  L.inv = take(R * 4);
  L.sorted_token = take(R * 4);
  // fp16 activations: T rows (decode path) or R expert-sorted rows (tensor-core path)
  L.x16 = take(R * d.hidden * 2);
  L.x_scale = take(R * 4);
  L.h = take(R * d.intermediate * 2);
  L.down_rows = take(R * d.hidden * 2);
  // LoRA-A products: fp32 [R, rank] for the GEMV path, fp16 [R, 64] for the tensor-core path
  const size_t xa_bytes = d.lora_rank > 0 ? (R * d.lora_rank * 4 > R * 128 ? R * d.lora_rank * 4 : R * 128) : 0;
  L.xa_gu = take(xa_bytes);
  L.xa_dn = take(xa_bytes);
  L.umma = take(umma_workspace_bytes(d.tokens, d.top_k, d.num_experts, d.hidden, d.intermediate));
  L.sync = take(decode_layer_sync_bytes(1024));
  L.part = take(decode_slice_shape(d) ? decode_slice_part_bytes(d) : 0);
  L.perm = take(permute_scratch_bytes(R, d.num_experts));
  L.total = o;
  return L;
}

__global__ void __launch_bounds__(256) convert_kernel(ConvertArgs c) {
  convert_rows_to_f16(c.src, c.src_dtype, c.dst, c.scale, c.rows, c.K, blockIdx.x * 8 + (threadIdx.x >> 5),
                      gridDim.x * 8);
}

// As convert_kernel, but row r of the output is source row rows_map[r].
__global__ void __launch_bounds__(256) gather_convert_kernel(ConvertArgs c, const int32_t* __restrict__ rows_map) {
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < c.rows; r += gridDim.x * 8) {
    const int64_t src = rows_map[r];
    convert_rows_to_f16(reinterpret_cast<const char*>(c.src) + src * c.K * 2, c.src_dtype, c.dst + (int64_t)r * c.K,
                        c.scale + r, 1, c.K, 0, 1);
  }
}

e4b_status launch_gather_convert(const ConvertArgs& c, const int32_t* rows_map, cudaStream_t s) {
  if (c.rows <= 0) return E4B_OK;
  gather_convert_kernel<<<conv_ctas_for(c.rows, 8), 256, 0, s>>>(c, rows_map);
  return launch_status();
}

__global__ void __launch_bounds__(256) gather_rows16_kernel(const uint4* __restrict__ src,
                                                            const int32_t* __restrict__ map, int rows, int vec,
                                                            uint4* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    const uint4* a = src + (int64_t)map[r] * vec;
    uint4* b = dst + (int64_t)r * vec;
    for (int v = lane; v < vec; v += 32) b[v] = a[v];
  }
}

e4b_status launch_gather_rows16(const void* src, const int32_t* rows_map, int rows, int K, void* dst, cudaStream_t s) {
  if (rows <= 0) return E4B_OK;
  int c = (rows + 7) / 8;
  c = c > 148 * 8 ? 148 * 8 : c;
  gather_rows16_kernel<<<c, 256, 0, s>>>(static_cast<const uint4*>(src), rows_map, rows, K / 8,
                                         static_cast<uint4*>(dst));
  return launch_status();
}

e4b_status check_weight_format(const e4b_moe_desc& d) {
  if (d.weight_format == E4B_FMT_NF4) return E4B_OK;
  if (d.weight_format == E4B_FMT_MXFP4) {  // bf16 compute on the tensor cores, whole 128-wide tiles
    if (d.lora_rank != 0 || d.act_dtype != E4B_BF16) return E4B_ERR_UNSUPPORTED;
    if (d.hidden % 128 || d.intermediate % 128) return E4B_ERR_UNSUPPORTED;
    return E4B_OK;
  }
  if (d.weight_format != E4B_FMT_FP8_BLOCK128) return E4B_ERR_INVALID_ARG;
  // FP8 experts: whole 128x128 scale tiles, no adapters
  if (d.lora_rank != 0) return E4B_ERR_UNSUPPORTED;
  if (d.hidden % 128 || d.intermediate % 128) return E4B_ERR_UNSUPPORTED;
  return E4B_OK;
}

int conv_ctas_for(int rows, int warps_per_cta) {
  int c = (rows + warps_per_cta - 1) / warps_per_cta;
  return c < 1 ? 1 : (c > 148 * 4 ? 148 * 4 : c);
}

// tile_start[e] = sum over e' < e of ceil(count(e') / tile_rows), one block of 1024 threads.
__global__ void __launch_bounds__(1024) tiles_from_offsets_kernel(const int32_t* __restrict__ offsets, int E,
                                                                  int tile_rows, int32_t* __restrict__ tile_start) {
  using Scan = cub::BlockScan<int, 1024>;
  __shared__ typename Scan::TempStorage tmp;
  const int e = threadIdx.x;
  const int c = e < E ? offsets[e + 1] - offsets[e] : 0;
  int ex, total;
  Scan(tmp).ExclusiveSum(c > 0 ? (c + tile_rows - 1) / tile_rows : 0, ex, total);
  if (e < E) tile_start[e] = ex;
  if (e == 0) tile_start[E] = total;
}

__global__ void active_from_offsets_kernel(const int32_t* __restrict__ offsets, int E, int32_t* __restrict__ active,
                                           int32_t* __restrict__ num_active) {
  if (threadIdx.x == 0) {
    int n = 0;
    for (int e = 0; e < E; ++e)
      if (offsets[e + 1] > offsets[e]) active[n++] = e;
    *num_active = n;
  }
}

void mark_stage(const e4b_moe_tensors* t, int i, cudaStream_t s) {
  if (!t->stage_events || !t->stage_events[i]) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cs);
  cudaEvent_t ev = (cudaEvent_t)t->stage_events[i];
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, s);
}

e4b_status run_expert_stages(const e4b_moe_desc& d, const e4b_moe_tensors* t, const ExpertRows& x, cudaStream_t s) {
  const int E = d.num_experts, H = d.hidden, I = d.intermediate, R = x.R;
  const int n1 = d.has_gate ? 2 * I : I;
  const int max_active = R < E ? R : E;
  const int lora_tiles = R / kLoraRows + max_active;
  e4b_status st = E4B_OK;
  if (d.weight_format == E4B_FMT_MXFP4) {
    // bf16 activation rows (expert-sorted), bf16 h and down rows: the reference's bf16 lane
    GemvArgs g{};
    g.a = x.x16;  // bf16 bytes in the same buffer
    g.packed = t->gate_up_packed;
    g.absmax = t->gate_up_absmax;  // e8m0 bytes
    g.offsets = x.offsets;
    g.active = x.active;
    g.num_active = x.num_active;
    g.E = E;
    g.N = n1;
    g.K = H;
    g.epilogue = d.has_gate ? E4B_EPI_SWIGLU : E4B_EPI_SILU;
    g.out = x.h;
    g.out_dtype = E4B_BF16;
    g.Nout = I;
    g.tiles_per_expert = I / 16;
    g.max_tasks = max_active * g.tiles_per_expert;
    g.err = x.err;
    mark_stage(t, 2, s);
    if ((st = launch_umma(umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R), d.act_dtype, s, E4B_FMT_MXFP4)) !=
        E4B_OK)
      return st;
    mark_stage(t, 3, s);
    mark_stage(t, 4, s);
    g.a = x.h;
    g.packed = t->down_packed;
    g.absmax = t->down_absmax;
    g.N = H;
    g.K = I;
    g.epilogue = E4B_EPI_NONE;
    g.out = x.down_rows;
    g.Nout = H;
    g.tiles_per_expert = H / 16;
    g.max_tasks = max_active * g.tiles_per_expert;
    if ((st = launch_umma(umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R), d.act_dtype, s, E4B_FMT_MXFP4)) !=
        E4B_OK)
      return st;
    mark_stage(t, 5, s);
    return E4B_OK;
  }
  if (d.weight_format == E4B_FMT_FP8_BLOCK128) {
    mark_stage(t, 2, s);
    GemvArgs g{};
    g.a = x.x16;
    g.a_scale = x.x_scale;
    g.a_rows = x.a_rows;
    g.packed = t->gate_up_packed;
    g.absmax = t->gate_up_absmax;  // fp32 tile scales
    g.offsets = x.offsets;
    g.active = x.active;
    g.num_active = x.num_active;
    g.E = E;
    g.N = n1;
    g.K = H;
    g.epilogue = d.has_gate ? E4B_EPI_SWIGLU : E4B_EPI_SILU;
    g.out = x.h;
    g.out_dtype = E4B_F16;
    g.Nout = I;
    g.tiles_per_expert = I / 16;
    g.max_tasks = max_active * g.tiles_per_expert;
    g.err = x.err;
    if (x.use_umma)
      st = launch_umma(umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R), d.act_dtype, s, d.weight_format);
    else
      st = launch_fp8_gemv(g, s);
    if (st != E4B_OK) return st;
    mark_stage(t, 3, s);
    mark_stage(t, 4, s);
    g.a = x.h;
    g.a_scale = nullptr;
    g.a_rows = nullptr;
    g.packed = t->down_packed;
    g.absmax = t->down_absmax;
    g.N = H;
    g.K = I;
    g.epilogue = E4B_EPI_NONE;
    g.out = x.down_rows;
    g.out_dtype = E4B_F16;
    g.Nout = H;
    g.tiles_per_expert = H / 16;
    g.max_tasks = max_active * g.tiles_per_expert;
    if (x.use_umma)
      st = launch_umma(umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R), d.act_dtype, s, d.weight_format);
    else
      st = launch_fp8_gemv(g, s);
    if (st != E4B_OK) return st;
    mark_stage(t, 5, s);
    return E4B_OK;
  }
  if (d.lora_rank > 0) {
    LoraAArgs la{};
    la.a = x.x16;
    la.a_scale = x.x_scale;
    la.a_rows = x.a_rows;
    la.loraA = t->gate_up_lora_A;
    la.offsets = x.offsets;
    la.tile_start = x.tile_a;
    la.E = E;
    la.K = H;
    la.rank = d.lora_rank;
    la.lora_dtype = d.lora_dtype;
    la.scaling = d.lora_scaling;
    la.xa = x.xa_gu;
    if (x.use_umma) la.xa16 = reinterpret_cast<__half*>(x.xa_gu);
    la.max_tiles = lora_tiles;
    if ((st = launch_lora_a(la, s)) != E4B_OK) return st;
  }
  mark_stage(t, 2, s);

  GemvArgs g{};
  g.a = x.x16;
  g.a_scale = x.x_scale;
  g.a_rows = x.a_rows;
  g.packed = t->gate_up_packed;
  g.absmax = t->gate_up_absmax;
  g.offsets = x.offsets;
  g.active = x.active;
  g.num_active = x.num_active;
  g.E = E;
  g.N = n1;
  g.K = H;
  g.epilogue = d.has_gate ? E4B_EPI_SWIGLU : E4B_EPI_SILU;
  g.out = x.h;
  g.out_dtype = E4B_F16;
  g.Nout = I;
  g.lora_xa = d.lora_rank > 0 ? x.xa_gu : nullptr;
  g.lora_B = t->gate_up_lora_B;
  g.lora_dtype = d.lora_dtype;
  g.rank = d.lora_rank;
  g.tiles_per_expert = n1 / 16;
  g.max_tasks = max_active * g.tiles_per_expert;
  g.err = x.err;
  if (x.use_umma) {
    UmmaArgs u = umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R);
    u.lora_xa16 = reinterpret_cast<const __half*>(g.lora_xa);  // fp16 [R, 64] in the tensor-core path
    st = launch_umma(u, d.act_dtype, s);
  } else {
    st = launch_gemv_auto(g, x.x_rows, x.max_rows_per_expert, s);
  }
  if (st != E4B_OK) return st;
  mark_stage(t, 3, s);

  if (d.lora_rank > 0) {
    LoraAArgs la{};
    la.a = reinterpret_cast<const __half*>(x.h);
    la.a_scale = nullptr;
    la.a_rows = nullptr;
    la.loraA = t->down_lora_A;
    la.offsets = x.offsets;
    la.tile_start = x.tile_a;
    la.E = E;
    la.K = I;
    la.rank = d.lora_rank;
    la.lora_dtype = d.lora_dtype;
    la.scaling = d.lora_scaling;
    la.xa = x.xa_dn;
    if (x.use_umma) la.xa16 = reinterpret_cast<__half*>(x.xa_dn);
    la.max_tiles = lora_tiles;
    if ((st = launch_lora_a(la, s)) != E4B_OK) return st;
  }
  mark_stage(t, 4, s);

  g.a = x.h;
  g.a_scale = nullptr;
  g.a_rows = nullptr;
  g.packed = t->down_packed;
  g.absmax = t->down_absmax;
  g.N = H;
  g.K = I;
  g.epilogue = E4B_EPI_NONE;
  g.out = x.down_rows;
  g.out_dtype = E4B_F16;  // fp16 rows: one bf16 rounding (the final output) instead of two
  g.Nout = H;
  g.lora_xa = d.lora_rank > 0 ? x.xa_dn : nullptr;
  g.lora_B = t->down_lora_B;
  g.tiles_per_expert = H / 16;
  g.max_tasks = max_active * g.tiles_per_expert;
  if (x.use_umma) {
    UmmaArgs u = umma_args_from(g, x.umma_scratch, x.tile_b, R, 1, R);
    u.lora_xa16 = reinterpret_cast<const __half*>(g.lora_xa);  // fp16 [R, 64] in the tensor-core path
    st = launch_umma(u, d.act_dtype, s);
  } else {
    st = launch_gemv_auto(g, R, x.max_rows_per_expert, s);
  }
  if (st != E4B_OK) return st;
  mark_stage(t, 5, s);
  return E4B_OK;
}

static bool desc_ok(const e4b_moe_desc& d) {
  if (d.num_experts <= 0 || d.num_experts > 1024 || d.hidden <= 0 || d.intermediate <= 0) return false;
  if (d.top_k <= 0 || d.top_k > 32 || d.top_k > d.num_experts || d.tokens < 0) return false;
  if ((int64_t)d.tokens * d.top_k > (1 << 30)) return false;
  if (d.routed_experts < 0 || d.routed_experts > (1 << 24)) return false;
  return true;
}

}  // namespace e4b

using namespace e4b;

extern "C" const char* e4b_status_string(e4b_status s) {
  switch (s) {
    case E4B_OK: return "ok";
    case E4B_ERR_INVALID_ARG: return "invalid argument (null pointer or inconsistent sizes)";
    case E4B_ERR_UNSUPPORTED: return "unsupported configuration (dtype, blocksize, K % 64, or rank)";
    case E4B_ERR_WORKSPACE: return "workspace missing or too small";
    case E4B_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case E4B_ERR_CUDA: return "CUDA launch or query failed";
    case E4B_ERR_EXPERT_INDEX: return "top-k expert index outside [0, num_experts)";
    case E4B_ERR_RANGE: return "an intermediate activation exceeded the fp16 range (+-65504) and was saturated";
    case E4B_ERR_TIMEOUT: return "a bounded device wait (asynchronous copy or peer arrival flag) timed out";
    case E4B_ERR_STATIC_SCRATCH:
      return "layer needs more scratch than the static array of e4b_moe_forward_static (E4B_STATIC_SCRATCH_BYTES)";
  }
  return "unknown status";
}

extern "C" int e4b_abi_version(void) { return 4; }

extern "C" e4b_status e4b_read_device_error(void* workspace, void* stream, int* error_out) {
  if (!workspace || !error_out) return E4B_ERR_INVALID_ARG;
  cudaStream_t s = (cudaStream_t)stream;
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return E4B_ERR_CUDA;
  if (cudaMemsetAsync(workspace, 0, sizeof(int), s) != cudaSuccess) return E4B_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return E4B_ERR_CUDA;
  *error_out = v;
  return E4B_OK;
}

extern "C" int e4b_watch_device_error(void* workspace, int* host_word, void* event, void* stream) {
  if (!workspace || !host_word || !event) return 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaEvent_t ev = (cudaEvent_t)event;
  int prev = 0;
  const cudaError_t q = cudaEventQuery(ev);
  if (q == cudaSuccess) prev = *reinterpret_cast<volatile int*>(host_word);
  else if (q != cudaErrorNotReady) cudaGetLastError();  // an event never recorded yet
  if (cudaMemcpyAsync(host_word, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) == cudaSuccess)
    cudaEventRecord(ev, s);
  return prev;
}

extern "C" size_t e4b_grouped_gemm_workspace_bytes(int R, int E, int N, int K) {
  (void)N;
  if (E <= 0 || R < 0 || K <= 0) return 0;
  return kErrBytes + align_up((size_t)(E + 1) * 4, 256) + align_up((size_t)R * K * 2, 256) +
         align_up((size_t)R * 4, 256) + align_up((size_t)(E + 1) * 4, 256);
}

extern "C" e4b_status e4b_grouped_nf4_gemm(const void* a, int a_dtype, const int32_t* a_rows, const uint8_t* packed,
                                           const float* absmax, const int32_t* offsets, int E, int R, int N, int K,
                                           int epilogue, void* out, void* workspace, size_t workspace_bytes,
                                           void* stream) {
  if (E <= 0 || E > 1024 || R < 0 || N <= 0 || K <= 0) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(a_dtype) || K % 64) return E4B_ERR_UNSUPPORTED;
  if (epilogue == E4B_EPI_SWIGLU ? (N % 32) : (N % 16)) return E4B_ERR_UNSUPPORTED;
  if (epilogue < E4B_EPI_NONE || epilogue > E4B_EPI_SILU) return E4B_ERR_INVALID_ARG;
  if (R == 0) return E4B_OK;
  if (!a || !packed || !absmax || !offsets || !out) return E4B_ERR_INVALID_ARG;
  if (!aligned16(a) || !aligned16(packed)) return E4B_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < e4b_grouped_gemm_workspace_bytes(R, E, N, K)) return E4B_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int32_t* active = reinterpret_cast<int32_t*>(ws + kErrBytes);
  int32_t* num_active = reinterpret_cast<int32_t*>(ws + 4);  // second word of the error block
  __half* a16 = reinterpret_cast<__half*>(ws + kErrBytes + align_up((size_t)(E + 1) * 4, 256));
  float* a_scale = reinterpret_cast<float*>(reinterpret_cast<char*>(a16) + align_up((size_t)R * K * 2, 256));
  active_from_offsets_kernel<<<1, 32, 0, s>>>(offsets, E, active, num_active);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  // source rows of `a`: R rows, or (with a gather map) up to max(a_rows)+1 -- converted lazily
  // by converting R rows of the gathered order into a16 and dropping the map.
  ConvertArgs cv{};
  cv.src = a;
  cv.src_dtype = a_dtype;
  cv.dst = a16;
  cv.scale = a_scale;
  cv.rows = R;
  cv.K = K;
  if (a_rows) {
    gather_convert_kernel<<<conv_ctas_for(R, 8), 256, 0, s>>>(cv, a_rows);
  } else {
    convert_kernel<<<conv_ctas_for(R, 8), 256, 0, s>>>(cv);
  }
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  GemvArgs g{};
  g.a = a16;
  g.a_scale = a_scale;
  g.a_rows = nullptr;
  g.out_dtype = a_dtype;
  g.packed = packed;
  g.absmax = absmax;
  g.offsets = offsets;
  g.active = active;
  g.num_active = num_active;
  g.E = E;
  g.N = N;
  g.K = K;
  g.epilogue = epilogue;
  g.out = out;
  g.Nout = epilogue == E4B_EPI_SWIGLU ? N / 2 : N;
  g.tiles_per_expert = epilogue == E4B_EPI_SWIGLU ? N / 16 : N / 16;
  g.max_tasks = (R < E ? R : E) * g.tiles_per_expert;
  g.err = reinterpret_cast<int*>(ws);
  // Prefill-sized groups take the tcgen05 kernel (the same rule as the fused layer: at
  // least 16 rows per expert on average), with its 128-row token tiles counted here.
  const int n_out = epilogue == E4B_EPI_SWIGLU ? N / 2 : N;
  if (umma_worthwhile(R, E) && R > 16 && n_out % 128 == 0 && umma_eligible(R, 1, E, K, n_out, 1, a_dtype, 0)) {
    int32_t* tile_start = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(a_scale) + align_up((size_t)R * 4, 256));
    tiles_from_offsets_kernel<<<1, 1024, 0, s>>>(offsets, E, kUmmaTokens, tile_start);
    if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
    return launch_umma(umma_args_from(g, nullptr, tile_start, R, 1, R), a_dtype, s);
  }
  return launch_gemv_auto(g, R, R, s);
}

extern "C" size_t e4b_grouped_nf4_dgrad_workspace_bytes(int R, int E, int N, int K) {
  (void)K;
  if (E <= 0 || R < 0 || N <= 0) return 0;
  return kErrBytes + align_up((size_t)R * N * 2, 256) + align_up((size_t)R * 4, 256) +
         align_up((size_t)(E + 1) * 4, 256);
}

extern "C" e4b_status e4b_grouped_nf4_dgrad(const void* dy, int dy_dtype, const uint8_t* packed, const float* absmax,
                                            const int32_t* offsets, int E, int R, int N, int K, void* dx,
                                            int dx_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (E <= 0 || E > 1024 || R < 0 || N <= 0 || K <= 0) return E4B_ERR_INVALID_ARG;
  if (!is_act_dtype(dy_dtype) || !(dx_dtype == E4B_F32 || is_act_dtype(dx_dtype))) return E4B_ERR_UNSUPPORTED;
  if (!umma_dgrad_eligible(N, K)) return E4B_ERR_UNSUPPORTED;
  if (R == 0) return E4B_OK;
  if (!dy || !packed || !absmax || !offsets || !dx) return E4B_ERR_INVALID_ARG;
  if (!aligned16(dy) || !aligned16(packed) || !aligned16(dx)) return E4B_ERR_ALIGNMENT;
  if (!workspace || workspace_bytes < e4b_grouped_nf4_dgrad_workspace_bytes(R, E, N, K)) return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  __half* dy16 = reinterpret_cast<__half*>(ws + kErrBytes);
  float* dy_scale = reinterpret_cast<float*>(reinterpret_cast<char*>(dy16) + align_up((size_t)R * N * 2, 256));
  int32_t* tile_start = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(dy_scale) + align_up((size_t)R * 4, 256));
  ConvertArgs cv{};
  cv.src = dy;
  cv.src_dtype = dy_dtype;
  cv.dst = dy16;
  cv.scale = dy_scale;
  cv.rows = R;
  cv.K = N;
  convert_kernel<<<conv_ctas_for(R, 8), 256, 0, s>>>(cv);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  tiles_from_offsets_kernel<<<1, 1024, 0, s>>>(offsets, E, kUmmaTokens, tile_start);
  if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  GemvArgs g{};
  g.a = dy16;
  g.a_scale = dy_scale;
  g.packed = packed;
  g.absmax = absmax;
  g.offsets = offsets;
  g.E = E;
  g.N = N;
  g.K = K;
  g.epilogue = E4B_EPI_NONE;
  g.out = dx;
  g.out_dtype = dx_dtype;
  g.Nout = K;
  g.err = reinterpret_cast<int*>(ws);
  return launch_umma_dgrad(umma_args_from(g, nullptr, tile_start, R, 1, R), dx_dtype, s);
}

extern "C" size_t e4b_moe_decode_step_workspace_bytes(const e4b_moe_desc* desc) {
  if (!desc || !desc_ok(*desc)) return 0;
  return align_up(moe_layout(*desc).total, 256) + e4b_router_workspace_bytes(desc->tokens, desc->num_experts);
}

extern "C" e4b_status e4b_moe_decode_step(const e4b_moe_desc* desc, const e4b_moe_tensors* t, const void* router_w,
                                          int router_w_dtype, int kind, int norm_topk_prob, int64_t* topk_idx,
                                          float* topk_w, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc || !t || !desc_ok(*desc)) return E4B_ERR_INVALID_ARG;
  if (!router_w || !topk_idx || !topk_w) return E4B_ERR_INVALID_ARG;
  if (t->expert_map || desc->routed_experts) return E4B_ERR_UNSUPPORTED;  // the router scores every stack row
  if (!is_any_dtype(router_w_dtype)) return E4B_ERR_UNSUPPORTED;
  if (kind != E4B_SOFTMAX_THEN_TOPK && kind != E4B_TOPK_THEN_SOFTMAX) return E4B_ERR_INVALID_ARG;
  const size_t need = e4b_moe_decode_step_workspace_bytes(desc);
  if (!workspace || workspace_bytes < need) return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace) || !aligned16(router_w)) return E4B_ERR_ALIGNMENT;
  e4b_moe_desc d = *desc;
  d.weight_dtype = E4B_F32;  // the router's weights
  e4b_moe_tensors tt = *t;
  tt.topk_idx = topk_idx;
  tt.topk_w = topk_w;
  char* ws = static_cast<char*>(workspace);
  const size_t layer_bytes = align_up(moe_layout(d).total, 256);
  char* rws = ws + layer_bytes;
  cudaStream_t s = (cudaStream_t)stream;
  const bool tensors_ok = t->hidden && t->out && t->gate_up_packed && t->gate_up_absmax && t->down_packed &&
                          t->down_absmax && aligned16(t->hidden) && aligned16(t->out) &&
                          aligned16(t->gate_up_packed) && aligned16(t->down_packed) &&
                          aligned16(t->gate_up_absmax) && aligned16(t->down_absmax) && is_act_dtype(d.act_dtype) &&
                          is_any_dtype(d.out_dtype);
  if (d.tokens > 0 && tensors_ok && decode_flow_eligible(d, true)) {
    const MoeLayout L = moe_layout(d);
    DecodeRouter r{router_w, router_w_dtype, kind, norm_topk_prob, topk_idx, topk_w, nullptr};
    mark_stage(&tt, 0, s);
    e4b_status st = launch_decode_flow(d, &tt, ws + L.h, ws + kFlowSyncOffset, reinterpret_cast<int*>(ws), s, &r);
    for (int i = 1; i < E4B_MOE_STAGE_EVENTS; ++i) mark_stage(&tt, i, s);
    return st;
  }
  if (d.tokens > 0 && tensors_ok && decode_layer_eligible(d) && decode_router_fusable(d)) {
    const MoeLayout L = moe_layout(d);
    DecodeRouter r{router_w, router_w_dtype, kind, norm_topk_prob, topk_idx, topk_w,
                   reinterpret_cast<float*>(rws + kErrBytes)};
    mark_stage(&tt, 0, s);
    e4b_status st = launch_decode_layer(d, &tt, ws + L.h, ws + L.down_rows, ws + L.sync, reinterpret_cast<int*>(ws), s,
                                        &r, decode_slice_shape(d) ? ws + L.part : nullptr);
    for (int i = 1; i < E4B_MOE_STAGE_EVENTS; ++i) mark_stage(&tt, i, s);
    return st;
  }
  e4b_status st = e4b_router_topk(t->hidden, d.act_dtype, router_w, router_w_dtype, d.tokens, d.hidden, d.num_experts,
                                  d.top_k, kind, norm_topk_prob, nullptr, topk_idx, topk_w, rws,
                                  e4b_router_workspace_bytes(d.tokens, d.num_experts), stream);
  if (st != E4B_OK) return st;
  return e4b_moe_forward(&d, &tt, workspace, layer_bytes, stream);
}

extern "C" int e4b_moe_path(const e4b_moe_desc* desc) {
  if (!desc || !desc_ok(*desc)) return -1;
  const e4b_moe_desc& d = *desc;
  if (decode_flow_eligible(d, false) || decode_layer_eligible(d)) return E4B_PATH_DECODE_LAYER;
  if (d.weight_format == E4B_FMT_MXFP4) return E4B_PATH_TENSOR_CORE;
  const int64_t R = (int64_t)d.tokens * d.top_k;
  if (umma_worthwhile(R, d.num_experts) &&
      umma_eligible(d.tokens, d.top_k, d.num_experts, d.hidden, d.intermediate, d.has_gate, d.act_dtype, d.lora_rank))
    return E4B_PATH_TENSOR_CORE;
  return E4B_PATH_STREAMING;
}

extern "C" size_t e4b_moe_workspace_bytes(const e4b_moe_desc* desc) {
  if (!desc || !desc_ok(*desc)) return 0;
  return moe_layout(*desc).total;
}

extern "C" e4b_status e4b_moe_forward(const e4b_moe_desc* desc, const e4b_moe_tensors* t, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (!desc || !t || !desc_ok(*desc)) return E4B_ERR_INVALID_ARG;
  const e4b_moe_desc& d = *desc;
  if (!is_act_dtype(d.act_dtype) || !is_any_dtype(d.weight_dtype) || !is_any_dtype(d.out_dtype))
    return E4B_ERR_UNSUPPORTED;
  if (d.hidden % 64 || d.intermediate % 64) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank < 0 || d.lora_rank > kLoraMaxRank) return E4B_ERR_UNSUPPORTED;
  if (d.lora_rank > 0 && !is_any_dtype(d.lora_dtype)) return E4B_ERR_UNSUPPORTED;
  if (e4b_status fs = check_weight_format(d)) return fs;
  const int T = d.tokens, k = d.top_k, E = d.num_experts, H = d.hidden, I = d.intermediate;
  if (T == 0) return E4B_OK;
  if (!t->hidden || !t->topk_idx || !t->topk_w || !t->gate_up_packed || !t->gate_up_absmax || !t->down_packed ||
      !t->down_absmax || !t->out)
    return E4B_ERR_INVALID_ARG;
  if (d.lora_rank > 0 && (!t->gate_up_lora_A || !t->gate_up_lora_B || !t->down_lora_A || !t->down_lora_B))
    return E4B_ERR_INVALID_ARG;
  if ((d.routed_experts > 0) != (t->expert_map != nullptr)) return E4B_ERR_INVALID_ARG;
  if (!aligned16(t->hidden) || !aligned16(t->gate_up_packed) || !aligned16(t->down_packed) || !aligned16(t->out))
    return E4B_ERR_ALIGNMENT;
  const MoeLayout L = moe_layout(d);
  if (!workspace || workspace_bytes < L.total) return E4B_ERR_WORKSPACE;
  if (!aligned16(workspace)) return E4B_ERR_ALIGNMENT;
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = static_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws);
  const int R = T * k;

  mark_stage(t, 0, s);
  if (decode_flow_eligible(d, false) && aligned16(t->gate_up_absmax) && aligned16(t->down_absmax)) {
    e4b_status st = launch_decode_flow(d, t, ws + L.h, ws + kFlowSyncOffset, err, s);  // one launch
    for (int i = 1; i < E4B_MOE_STAGE_EVENTS; ++i) mark_stage(t, i, s);
    return st;
  }
  if (decode_layer_eligible(d)) {  // one launch: permute, both GEMVs and the combine
    e4b_status st = launch_decode_layer(d, t, ws + L.h, ws + L.down_rows, ws + L.sync, err, s, nullptr,
                                        decode_slice_shape(d) ? ws + L.part : nullptr);
    for (int i = 1; i < E4B_MOE_STAGE_EVENTS; ++i) mark_stage(t, i, s);
    return st;
  }
  PermuteArgs pa{};
  pa.topk_idx = t->topk_idx;
  pa.T = T;
  pa.k = k;
  pa.E = E;
  pa.emap = t->expert_map;
  pa.routed = d.routed_experts;
  pa.inv = reinterpret_cast<int32_t*>(ws + L.inv);
  pa.sorted_token = reinterpret_cast<int32_t*>(ws + L.sorted_token);
  pa.offsets = reinterpret_cast<int32_t*>(ws + L.offsets);
  pa.active = reinterpret_cast<int32_t*>(ws + L.active);
  pa.num_active = reinterpret_cast<int32_t*>(ws + L.num_active);
  pa.tile_start_a = reinterpret_cast<int32_t*>(ws + L.tile_a);
  pa.tile_start_b = reinterpret_cast<int32_t*>(ws + L.tile_b);
  pa.tile_a = kLoraRows;
  pa.tile_b = kUmmaTokens;
  pa.err = err;
  if (permute_scratch_bytes((int64_t)T * k, E)) pa.seg_scratch = reinterpret_cast<int32_t*>(ws + L.perm);
  pa.reset_err = 0;  // the error word is sticky: only e4b_read_device_error clears it
  __half* x16 = reinterpret_cast<__half*>(ws + L.x16);
  float* x_scale = reinterpret_cast<float*>(ws + L.x_scale);
  pa.conv.src = t->hidden;
  pa.conv.src_dtype = d.act_dtype;
  pa.conv.dst = x16;
  pa.conv.scale = x_scale;
  pa.conv.rows = T;
  pa.conv.K = H;
  pa.conv_ctas = conv_ctas_for(T, 32);
  const bool mxfp4 = d.weight_format == E4B_FMT_MXFP4;
  const bool use_umma = mxfp4 || (umma_worthwhile((int64_t)T * k, E) &&
                                  umma_eligible(T, k, E, H, I, d.has_gate, d.act_dtype, d.lora_rank));
  if (use_umma) pa.conv.src = nullptr;  // converted below, in expert-sorted order
  e4b_status st = launch_permute(pa, s);
  if (st != E4B_OK) return st;
  if (mxfp4) {  // xs[r] = x[sorted_token[r]] as is (bf16): the bf16 tensor-core operand
    if ((st = launch_gather_rows16(t->hidden, pa.sorted_token, R, H, x16, s)) != E4B_OK) return st;
  } else if (use_umma) {  // xs[r] = fp16(x[sorted_token[r]]): contiguous rows per expert for the TMA tiles
    ConvertArgs cv{};
    cv.src = t->hidden;
    cv.src_dtype = d.act_dtype;
    cv.dst = x16;
    cv.scale = x_scale;
    cv.rows = R;
    cv.K = H;
    gather_convert_kernel<<<conv_ctas_for(R, 8), 256, 0, s>>>(cv, pa.sorted_token);
    if (launch_status() != E4B_OK) return E4B_ERR_CUDA;
  }
  mark_stage(t, 1, s);

  ExpertRows x{};
  x.x16 = x16;
  x.x_scale = x_scale;
  x.a_rows = use_umma ? nullptr : pa.sorted_token;
  x.x_rows = use_umma ? R : T;
  x.R = R;
  x.max_rows_per_expert = T;
  x.offsets = pa.offsets;
  x.active = pa.active;
  x.num_active = pa.num_active;
  x.tile_a = pa.tile_start_a;
  x.tile_b = pa.tile_start_b;
  x.use_umma = use_umma;
  x.h = ws + L.h;
  x.down_rows = ws + L.down_rows;
  x.xa_gu = reinterpret_cast<float*>(ws + L.xa_gu);
  x.xa_dn = reinterpret_cast<float*>(ws + L.xa_dn);
  x.umma_scratch = ws + L.umma;
  x.err = err;
  if ((st = run_expert_stages(d, t, x, s)) != E4B_OK) return st;

  st = e4b_combine(x.down_rows, mxfp4 ? E4B_BF16 : E4B_F16, pa.inv, t->topk_w, d.weight_dtype, T, k, H, t->out,
                   d.out_dtype, stream);
  mark_stage(t, 6, s);
  return st;
}
