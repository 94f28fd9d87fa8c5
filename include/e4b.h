/*
 * e4b.h -- C ABI of the B200 fused-expert library (libe4b.so).
 *
 * The reference (experts4bit-qlora) has no C ABI: its kernel boundary is a
 * Python call into grouped-nf4-gemm / bitsandbytes. Each entry point below
 * replaces one such call (or one stage of experts4bit_qlora/engines/fast.py)
 * and is cited to the reference line it stands in for. A maintainer binds them
 * with ctypes; the Python package in this repository does exactly that.
 *
 * Conventions
 *   - Every pointer is a DEVICE pointer unless the name ends in _host.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call is stream-ordered, never synchronises the host, and is
 *     therefore capturable in a CUDA graph. The library allocates nothing.
 *   - Return codes, never exceptions or device traps. Invalid expert ids found
 *     on the device are clamped for memory safety and reported through the
 *     device error word at the start of the workspace (e4b_read_device_error).
 *   - Layouts are the reference's storage contract
 *     (experts4bit_qlora/_vendor/experts.py:244-269): per expert, row-major
 *     [out, in] NF4 with two codes per byte (first element in the high nibble)
 *     and one fp32 absmax per 64 consecutive elements.
 */
#ifndef E4B_H_
#define E4B_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define E4B_API __attribute__((visibility("default")))
#else
#define E4B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  E4B_OK = 0,
  E4B_ERR_INVALID_ARG = 1,    /* null pointer, negative or inconsistent size */
  E4B_ERR_UNSUPPORTED = 2,    /* dtype / blocksize / K%64 / rank outside what the kernels take */
  E4B_ERR_WORKSPACE = 3,      /* workspace missing or smaller than *_workspace_bytes() */
  E4B_ERR_ALIGNMENT = 4,      /* a pointer is not 16-byte aligned */
  E4B_ERR_CUDA = 5,           /* a CUDA launch or query failed */
  E4B_ERR_EXPERT_INDEX = 6,   /* device-reported: a top-k index outside [0, E) */
  E4B_ERR_RANGE = 7,          /* device-reported: an intermediate activation beyond +-65504 saturated */
  E4B_ERR_TIMEOUT = 8,        /* device-reported: a bounded wait (async copy, peer flag) gave up */
  E4B_ERR_STATIC_SCRATCH = 9  /* layer needs more scratch than e4b_moe_forward_static's fixed array */
} e4b_status;

typedef enum { E4B_BF16 = 0, E4B_F16 = 1, E4B_F32 = 2 } e4b_dtype;

typedef enum {
  E4B_SOFTMAX_THEN_TOPK = 0,  /* OLMoE / Qwen3-MoE / Mixtral */
  E4B_TOPK_THEN_SOFTMAX = 1   /* gpt-oss */
} e4b_router_kind;

typedef enum { E4B_EPI_NONE = 0, E4B_EPI_SWIGLU = 1, E4B_EPI_SILU = 2 } e4b_epilogue;

/* Expert weight storage of the fused layer.
 * E4B_FMT_NF4: blockwise NF4 (2 codes per byte, first element in the high nibble)
 *   with one fp32 absmax per 64 consecutive elements (_vendor/experts.py:398-457).
 * E4B_FMT_FP8_BLOCK128: float8_e4m3fn bytes [out, in] per expert with one fp32
 *   multiplier per [128, 128] tile, [ceil(out/128), ceil(in/128)] per expert, the
 *   storage of formats/fp8_blocks.py:60-128 (an e8m0 scale is passed as its value
 *   2^(b-127)). The fused layer uses the weights at full precision, fp32(w) * scale.
 * E4B_FMT_MXFP4: OCP microscaling FP4, the storage of formats/mxfp4.py and of the
 *   reference's MXFP4 experts (engines/nvme_experts.py:769-868): e2m1 codes, two per
 *   byte, LOW nibble first, [E, out, in/2] bytes, and one e8m0 exponent byte per 32
 *   consecutive elements, [E, out, in/32] (passed in the *_absmax pointers). The
 *   layer computes in bf16 (act_dtype E4B_BF16; code * 2^(s-127) is exact in bf16),
 *   takes no adapters and needs hidden and intermediate % 128 == 0. */
typedef enum { E4B_FMT_NF4 = 0, E4B_FMT_FP8_BLOCK128 = 1, E4B_FMT_MXFP4 = 2 } e4b_weight_format;

E4B_API const char* e4b_status_string(e4b_status s);
/* ABI version: bumped when a signature or a struct below changes. */
E4B_API int e4b_abi_version(void);

/* ---- NF4 codec ---------------------------------------------------------- */

/* Replaces bitsandbytes.functional.quantize_4bit(w, blocksize=64,
 * compress_statistics=False, quant_type="nf4") as called per expert by
 * ExpertsNbit._quantize_stack (_vendor/experts.py:408-426). n % 64 == 0.
 * w: n elements of `w_dtype`; packed: n/2 bytes; absmax: n/64 fp32. */
E4B_API e4b_status e4b_nf4_quantize(const void* w, int w_dtype, int64_t n, uint8_t* packed, float* absmax,
                            void* stream);

/* Replaces bitsandbytes.functional.dequantize_4bit as called by
 * ExpertsNbit._dequantize_expert (_vendor/experts.py:447-457):
 * out[i] = out_dtype(code[q_i] * absmax[i/64]) with one round-to-nearest-even.
 * packed and out 16-byte aligned. */
E4B_API e4b_status e4b_nf4_dequantize(const uint8_t* packed, const float* absmax, int64_t n, void* out, int out_dtype,
                              void* stream);

/* Host (CPU) versions of the two calls above for modules built on CPU; they
 * produce the same bytes as the device kernels. */
E4B_API e4b_status e4b_nf4_quantize_host(const void* w_host, int w_dtype, int64_t n, uint8_t* packed_host,
                                 float* absmax_host);
E4B_API e4b_status e4b_nf4_dequantize_host(const uint8_t* packed_host, const float* absmax_host, int64_t n,
                                   void* out_host, int out_dtype);

/* ---- Router (R1) --------------------------------------------------------- */

/* Replaces transformers' OlmoeTopKRouter.forward (F.linear + fp32 softmax +
 * topk + optional renorm) with the rule of engines/cpu_router.py:100-119:
 * fp32 logits, stable descending order with ties to the LOWER expert id.
 * x [T,H] (x_dtype bf16/f16), w_router [E,H] (w_dtype bf16/f16/f32).
 * logits_out [T,E] fp32 is optional (NULL); topk_idx [T,k] int64; topk_w [T,k] fp32.
 * E <= 1024, k <= 32, k <= E. workspace: e4b_router_workspace_bytes(T,E). */
E4B_API size_t e4b_router_workspace_bytes(int T, int E);
E4B_API e4b_status e4b_router_topk(const void* x, int x_dtype, const void* w_router, int w_dtype, int T, int H, int E,
                           int k, int kind, int norm_topk_prob, float* logits_out, int64_t* topk_idx,
                           float* topk_w, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Permutation (R2) ---------------------------------------------------- */

/* Replaces engines/fast.py:126-135 (stable argsort of the flat indices,
 * bincount, nonzero, and the two .tolist() host syncs) with one device pass.
 * order [T*k]: order[r] = flat index (t*k+s) of sorted row r, stable within an
 * expert; inv [T*k]: inv[t*k+s] = r; offsets [E+1]: row start of each expert.
 * Any of order/inv may be NULL. workspace: e4b_permute_workspace_bytes. */
E4B_API size_t e4b_permute_workspace_bytes(int T, int k, int E);
E4B_API e4b_status e4b_permute(const int64_t* topk_idx, int T, int k, int E, int32_t* order, int32_t* inv,
                       int32_t* offsets, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Block-scaled FP8 weights (R12) -------------------------------------
 * dequantize_fp8_blocks (formats/fp8_blocks.py:60-128): out[o, i] =
 * dtype(fp32(e4m3 w[o, i]) * scale[o / 128, i / 128]); `scale` holds fp32 values
 * [ceil(rows/128), ceil(cols/128)]; ragged final tiles are allowed. */
E4B_API e4b_status e4b_fp8_block_dequantize(const uint8_t* w, const float* scale, int64_t rows, int64_t cols,
                                    void* out, int out_dtype, void* stream);

/* ---- MXFP4 weights (the storage format) ------------------------------------
 * Replaces formats/mxfp4.py:35-105 (dequantize_mxfp4): blocks uint8 [P, rows, G, B]
 * (two e2m1 codes per byte, low nibble first), scales uint8 [P, rows, G] (e8m0,
 * bias 127, one per block of 2B values); out [P, G*2B, rows] in out_dtype -- the
 * trailing (rows, K) pair transposed, as the reference returns it -- with
 * out = out_dtype(fp32(e2m1) * 2^(s-127)), one rounding. P = the product of the
 * leading dimensions (1 for a single projection). The _host variant takes host
 * pointers and produces the same bits. */
E4B_API e4b_status e4b_mxfp4_dequantize(const uint8_t* blocks, const uint8_t* scales, int64_t P, int64_t rows,
                                int64_t G, int64_t B, void* out, int out_dtype, void* stream);
E4B_API e4b_status e4b_mxfp4_dequantize_host(const uint8_t* blocks_host, const uint8_t* scales_host, int64_t P,
                                     int64_t rows, int64_t G, int64_t B, void* out_host, int out_dtype);

/* ---- Grouped NF4 GEMM (R3, R4, R6) --------------------------------------- */

/* Replaces nf4_grouped.gemm_4bit_grouped(a, packed.view(E,N,K/2),
 * absmax.view(E,N,K/64), sizes, expert_ids) (engines/fast.py:137-156) and,
 * with epilogue = E4B_EPI_SWIGLU, lora._epilogue (lora.py:102-128) fused on it.
 * a [R,K] (a_dtype bf16/f16): rows grouped by expert, expert e owning rows
 * [offsets[e], offsets[e+1]); with a_rows != NULL, row r is read from
 * a[a_rows[r]] instead (the permutation gather of fast.py:135 fused in).
 * out [R, N_out] in a_dtype, N_out = N/2 for SWIGLU (silu(gate)*up, gate = rows
 * [0, N/2)), else N. K % 64 == 0, N % 16 == 0 (N % 32 for SWIGLU).
 * workspace: e4b_grouped_gemm_workspace_bytes. */
E4B_API size_t e4b_grouped_gemm_workspace_bytes(int R, int E, int N, int K);
E4B_API e4b_status e4b_grouped_nf4_gemm(const void* a, int a_dtype, const int32_t* a_rows, const uint8_t* packed,
                                const float* absmax, const int32_t* offsets, int E, int R, int N, int K,
                                int epilogue, void* out, void* workspace, size_t workspace_bytes,
                                void* stream);

/* Replaces the single-launch dgrad kernel of grouped-nf4-gemm >= 0.7.0 that
 * fused_grouped_lora's backward calls with dgrad_kernel=True
 * (engines/fast.py:519-550, :453-552): the input gradient of a frozen grouped
 * projection, dx[r, :] = dy[r, :] . W_e for the rows r of expert e, with W_e the
 * NF4 stack packed [E, N, K/2], absmax [E, N, K/64] and no decoded stack in
 * memory. dy [R, N] (bf16/f16) rows grouped by expert as offsets [E+1]
 * (int32, device); dx [R, K] in dx_dtype (f32, bf16 or f16). N % 64 == 0,
 * K % 256 == 0. fp32 accumulation on the tensor cores (dy as fp16 under a
 * per-row power-of-two scale). workspace: e4b_grouped_nf4_dgrad_workspace_bytes. */
E4B_API size_t e4b_grouped_nf4_dgrad_workspace_bytes(int R, int E, int N, int K);
E4B_API e4b_status e4b_grouped_nf4_dgrad(const void* dy, int dy_dtype, const uint8_t* packed, const float* absmax,
                                 const int32_t* offsets, int E, int R, int N, int K, void* dx, int dx_dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- Combine (R7) -------------------------------------------------------- */

/* Replaces engines/fast.py:158-160 + _scatter_combine (:260-278): out[t] =
 * sum over s = 0..k-1 (in slot order, fp32) of w[t,s] * rows[inv[t*k+s]].
 * rows [T*k, H] (rows_dtype bf16, f16 or f32), w [T,k] (w_dtype; NULL: every
 * weight 1, the slot sum of the training backward's dL/dx), out [T,H] (out_dtype).
 * No atomics: bit-identical across runs. */
E4B_API e4b_status e4b_combine(const void* rows, int rows_dtype, const int32_t* inv, const void* w, int w_dtype, int T,
                       int k, int H, void* out, int out_dtype, void* stream);

/* ---- Training path element-wise steps (fast.py:453-552) ------------------ */

/* The differentiable layer of enable_fast_train (engines/fast.py:453-552) between its
 * grouped GEMMs, each one pass over the expert-sorted rows (replacing the torch
 * element-wise chains the reference runs there):
 * e4b_swiglu_forward: h [R, I] = act(gate) * up of proj [R, 2I] (has_gate; gate =
 *   columns [0, I)) or act(proj) [R, I], act = SiLU rounded to the dtype as
 *   lora._epilogue (lora.py:102-128) computes it; bf16/f16.
 * e4b_swiglu_backward: dproj [R, 2I] (or [R, I]) from dL/dh (fp32 [R, I]) and proj.
 * e4b_combine_row_grads: for the combine out[t] = sum_s w[t,s] down[row(t,s)], given
 *   dL/dout (fp32 [T, H]), the token of each sorted row (int64 [R]) and its weight
 *   (fp32 [R]): dd [R, H] = dL/dout[token] * w in the dtype, dw [R] = dL/dout[token] .
 *   down[r] in fp32 (the top-k weights' gradient, _scatter_combine :260-278). */
E4B_API e4b_status e4b_swiglu_forward(const void* proj, int dtype, int64_t R, int I, int has_gate, void* h,
                              void* stream);
E4B_API e4b_status e4b_swiglu_backward(const void* proj, int dtype, const float* dh, int64_t R, int I, int has_gate,
                               void* dproj, void* stream);
E4B_API e4b_status e4b_combine_row_grads(const float* grad, const int64_t* token_rows, const float* w_rows,
                                 const void* down, int dtype, int64_t R, int H, void* dd, float* dw,
                                 void* stream);

/* The rank-r adapter products of the same training path (lora.py:251-256 inside
 * fast.py:453-552), fp32 on expert-sorted rows with no padding of the experts'
 * segments (ranks 1..16). M_e(j, k) = M[e*sE + j*sj + k*sk] (fp32), so A [E, r, K]
 * and B [E, N, r] are read in either orientation. `tiles` [ntiles][3] int32 =
 * (expert, first row, rows <= 32); `segs` [nsegs][3] = (expert, first row, rows),
 * one per expert with rows.
 * e4b_lora_rank_down: Y [R, rk] = scale * X[row, :K] . M_e(j, :).
 * e4b_lora_rank_up: out[row, n] = scale * Y[row] . M_e(:, n) for n < N (mode 0, fp32
 *   out), += (mode 1, fp32), or out = dtype(out + dtype(delta)) (mode 2, bf16/f16).
 * e4b_lora_outer: G[e*gE + a*ga + j*gj] = scale * sum over e's rows of P[row, a] * Y[row, j]. */
E4B_API e4b_status e4b_lora_rank_down(const void* X, int x_dtype, int ldx, const float* M, int64_t sE, int64_t sj,
                              int64_t sk, int rk, int K, const int32_t* tiles, int ntiles, float scale, float* Y,
                              void* stream);
E4B_API e4b_status e4b_lora_rank_up(const float* Y, int rk, const float* M, int64_t sE, int64_t sj, int64_t sn, int N,
                            const int32_t* tiles, int ntiles, float scale, int mode, void* out, int out_dtype,
                            int ldo, void* stream);
E4B_API e4b_status e4b_lora_outer(const void* P, int p_dtype, int ldp, int A, const float* Y, int rk,
                          const int32_t* segs, int nsegs, float scale, float* G, int64_t gE, int64_t ga, int64_t gj,
                          void* stream);

/* ---- Whole expert layer (R2-R7 + LoRA R5) -------------------------------- */

typedef struct {
  int num_experts;        /* E */
  int hidden;             /* H: in-features of gate_up, out-features of down */
  int intermediate;       /* I: in-features of down */
  int top_k;              /* k */
  int tokens;             /* T */
  int has_gate;           /* 1: gate_up is [2I,H] (SwiGLU); 0: [I,H] (SiLU) */
  int act_dtype;          /* hidden / compute dtype: E4B_BF16 or E4B_F16 */
  int weight_dtype;       /* top_k_weights dtype: bf16 / f16 / f32 */
  int out_dtype;          /* output dtype (the caller's input dtype) */
  int lora_rank;          /* 0 = no adapter */
  int lora_dtype;         /* adapter dtype: E4B_F32 or E4B_BF16 (or E4B_F16) */
  float lora_scaling;     /* alpha / r */
  int weight_format;      /* e4b_weight_format; FP8 takes no adapters and needs H, I % 128 == 0 */
  /* Resident sub-stack (hot-expert residency, engines/hot_residency.py:39-104): 0 = the top-k ids
   * index the [E, ...] stacks directly; > 0 = the ids lie in [0, routed_experts) and
   * e4b_moe_tensors.expert_map[id] is the expert's index in the stacks (-1 = not resident,
   * reported as E4B_ERR_EXPERT_INDEX). Adapters are indexed the same way. */
  int routed_experts;
} e4b_moe_desc;

typedef struct {
  const void* hidden;              /* [T,H] act_dtype */
  const int64_t* topk_idx;         /* [T,k] */
  const void* topk_w;              /* [T,k] weight_dtype */
  const uint8_t* gate_up_packed;   /* [E, n1*H/2], n1 = 2I (has_gate) or I */
  const float* gate_up_absmax;     /* [E, n1*H/64] */
  const uint8_t* down_packed;      /* [E, H*I/2] */
  const float* down_absmax;        /* [E, H*I/64] */
  const void* gate_up_lora_A;      /* [E, r, H]   (NULL if lora_rank == 0) */
  const void* gate_up_lora_B;      /* [E, n1, r] */
  const void* down_lora_A;         /* [E, r, I] */
  const void* down_lora_B;         /* [E, H, r] */
  void* out;                       /* [T,H] out_dtype */
  /* Optional profiling hook (NULL normally): E4B_MOE_STAGE_EVENTS cudaEvent_t
   * handles recorded on `stream` before the permutation and after each of the
   * stages permute, LoRA-A(x), gate_up, LoRA-A(h), down, combine. While the
   * stream is being captured they are recorded as graph nodes, so a replayed
   * graph yields per-stage device times. */
  void* const* stage_events;
  const int32_t* expert_map;       /* [routed_experts] id -> stack index, or NULL (see routed_experts) */
} e4b_moe_tensors;

#define E4B_MOE_STAGE_EVENTS 7

/* Replaces fused_experts_forward / fused_experts_lora_forward
 * (engines/fast.py:100-160, :163-257) end to end: permutation, grouped
 * gate_up GEMM (+ LoRA delta before the activation) with SwiGLU, grouped down
 * GEMM (+ LoRA delta), weighted deterministic combine. No host sync. */
E4B_API size_t e4b_moe_workspace_bytes(const e4b_moe_desc* desc);
E4B_API e4b_status e4b_moe_forward(const e4b_moe_desc* desc, const e4b_moe_tensors* t, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Which kernel sequence e4b_moe_forward runs for `desc` (no counterpart in the
 * reference): E4B_PATH_DECODE_LAYER = one persistent launch for the whole layer
 * (decode regime, NF4, no adapters), E4B_PATH_STREAMING = permute + grouped GEMV
 * kernels, E4B_PATH_TENSOR_CORE = permute + tcgen05 grouped GEMMs; -1 for an
 * invalid descriptor. e4b_set_decode_kernel(0) turns the one-launch path off for
 * the process (also E4B_DECODE_KERNEL=0 in the environment); returns the
 * previous setting (-1 = not yet read). */
#define E4B_PATH_STREAMING 0
#define E4B_PATH_TENSOR_CORE 1
#define E4B_PATH_DECODE_LAYER 2
E4B_API int e4b_moe_path(const e4b_moe_desc* desc);
/* mode 0: no one-launch kernel; 1: the flow kernel (per-expert completion counters, up to 8
 * tokens and 64 picks) where it applies, else the phase kernel; 2: the phase kernel only
 * (grid-synchronised phases, up to 16 tokens and 128 picks); 3 (default): the slice kernel
 * (units of one expert x 64 intermediate columns, gated layers, up to 8 tokens, H a multiple
 * of 512) where it applies, else the phase kernel. Any other value selects 3. */
E4B_API int e4b_set_decode_kernel(int mode);

/* No counterpart in the reference (its router is the model's own module): router
 * and expert layer in one call. Top-k of fp32 logits x . W_r^T (router_w [E, H],
 * rules as e4b_router_topk) into topk_idx / topk_w (fp32), then the layer of
 * e4b_moe_forward with those picks (t->topk_idx / t->topk_w are ignored). In the
 * decode regime (E4B_PATH_DECODE_LAYER) both run in one launch; otherwise it
 * runs e4b_router_topk then e4b_moe_forward. Workspace:
 * e4b_moe_decode_step_workspace_bytes. */
E4B_API size_t e4b_moe_decode_step_workspace_bytes(const e4b_moe_desc* desc);
E4B_API e4b_status e4b_moe_decode_step(const e4b_moe_desc* desc, const e4b_moe_tensors* t, const void* router_w,
                               int router_w_dtype, int kind, int norm_topk_prob, int64_t* topk_idx, float* topk_w,
                               void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart in the reference. Same layer as e4b_moe_forward for callers
 * that cannot allocate device memory (a host framework that owns all device
 * allocations, a plugin host that forbids cudaMalloc after start-up): the
 * scratch is a fixed library-owned device array of E4B_STATIC_SCRATCH_BYTES
 * held on every GPU that loads the library. Layers needing more
 * (e4b_moe_workspace_bytes) are refused with E4B_ERR_STATIC_SCRATCH. The first
 * call on a device looks up the array's address and should come before any
 * stream capture there. All calls on a device share the array: calls that
 * overlap on the GPU race. Allocates nothing. */
#define E4B_STATIC_SCRATCH_BYTES (16u << 20)
E4B_API e4b_status e4b_moe_forward_static(const e4b_moe_desc* desc, const e4b_moe_tensors* t, void* stream);

/* ---- Expert parallelism (experts sharded over P ranks) ---------
 * No counterpart in the reference (it has no distributed code); the split
 * follows its per-expert loop (_vendor/experts.py:486-513). Rank p owns the
 * experts [p*E/P, (p+1)*E/P). One layer on every rank:
 *   1. e4b_ep_dispatch on the rank's token shard: stable permutation by global
 *      expert (as fast.py:125-135), rows gathered into send_rows [T*k, H] in that
 *      order, per-expert row counts [E] and the inverse permutation [T*k].
 *   2. caller: all-to-all of the counts (E/P per peer) and of the rows (the rows
 *      for peer q are send_rows[offsets[q*E/P] .. offsets[(q+1)*E/P])).
 *   3. e4b_ep_experts on the received rows (source-major): `local` describes the
 *      rank's experts (num_experts = E/P, top_k = 1, tokens = received rows,
 *      out_dtype = E4B_F16), `recv_counts` [P, E/P] (device), t->hidden = received
 *      rows, t->out = unweighted fp16 down rows [tokens, H] in the received order;
 *      t's weight/adapter pointers are the rank's expert slices. topk_* unused.
 *   4. caller: reverse all-to-all of those rows; they land in send_rows' order.
 *   5. e4b_combine(rows, E4B_F16, inv, topk_w, ...) on the shard. */
E4B_API size_t e4b_ep_dispatch_workspace_bytes(int T, int k, int E);
E4B_API e4b_status e4b_ep_dispatch(const void* hidden, int act_dtype, const int64_t* topk_idx, int T, int k, int E,
                           int H, void* send_rows, int32_t* expert_counts, int32_t* inv, void* workspace,
                           size_t workspace_bytes, void* stream);
E4B_API size_t e4b_ep_experts_workspace_bytes(const e4b_moe_desc* local, int world);
E4B_API e4b_status e4b_ep_experts(const e4b_moe_desc* local, int world, const int32_t* recv_counts,
                          const e4b_moe_tensors* t, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Expert parallelism over peer memory (one node, NVLink) -------
 * No counterpart in the reference (it has no distributed code). The same layer
 * as the section above, with both exchanges done by the library's own kernels
 * as stores into the other ranks' memory instead of the caller's all-to-alls,
 * so nothing waits on the host: no count exchange, no host sync, fixed shapes.
 *
 * Every rank owns one exchange region of e4b_ep_comm_bytes() bytes, zeroed
 * before first use, and maps every other rank's region (CUDA IPC:
 * e4b_ipc_export on the owner, e4b_ipc_open on the others). The region holds
 * an error word, arrival flags, the counts and rows each source sends
 * (rows_per_rank rows per source, in the source's expert-major order) and the
 * returned down rows of the rank's own picks. One layer, on every rank:
 *   1. e4b_ep_dispatch_peer: permutation + row gather; rows, per-expert counts
 *      and the send offset go straight into each owner's region, then the
 *      arrival flag (release at system scope).
 *   2. e4b_ep_experts_peer: waits (bounded) for every source's flag, plans the
 *      received rows, runs the expert stages, and stores the fp16 down rows
 *      into each source's region at that source's sorted position, then a flag.
 *   3. e4b_ep_combine_peer: waits (bounded) for every owner's flag and combines.
 * The region counts the layer calls it has completed (advanced on the device by
 * e4b_ep_combine_peer), and each step waits for its peers' flags to reach the
 * current call's number, so nothing changes on the host between calls and a
 * layer call can be captured in a CUDA graph and replayed. One region serves any
 * number of layers called in the same order on every rank. Waits give up after a
 * few seconds with E4B_ERR_TIMEOUT in the region's error word (sticky: read and
 * cleared with e4b_read_device_error(region, ...)). */
#define E4B_IPC_HANDLE_BYTES 64
#define E4B_EP_MAX_PEERS 16
typedef struct {
  int world;            /* ranks in the group, 1..E4B_EP_MAX_PEERS */
  int rank;             /* this rank */
  int local_experts;    /* E / world */
  int rows_per_rank;    /* capacity: the most T*k rows any rank dispatches in one layer */
  int hidden;           /* H, a multiple of 64 */
  int act_dtype;        /* dtype of the exchanged activation rows (E4B_BF16 or E4B_F16) */
  void* const* peers;   /* HOST array [world]: each rank's region as mapped here (peers[rank] = own) */
} e4b_ep_peer_desc;

E4B_API size_t e4b_ep_comm_bytes(int world, int local_experts, int rows_per_rank, int hidden);
/* Device memory <-> IPC handle (E4B_IPC_HANDLE_BYTES bytes) plus the offset of ptr in its allocation. */
E4B_API e4b_status e4b_ipc_export(const void* ptr, void* handle_host, size_t* offset_host);
E4B_API e4b_status e4b_ipc_open(const void* handle_host, size_t offset, void** ptr_host);
E4B_API e4b_status e4b_ipc_close(void* ptr, size_t offset);
E4B_API size_t e4b_ep_dispatch_peer_workspace_bytes(int T, int k, int E);
E4B_API e4b_status e4b_ep_dispatch_peer(const e4b_ep_peer_desc* pd, const void* hidden, const int64_t* topk_idx, int T,
                                int k, int32_t* inv, void* workspace, size_t workspace_bytes, void* stream);
/* local: the rank's experts as for e4b_ep_experts (top_k = 1, out_dtype = E4B_F16);
 * local->tokens = the rows this rank expects to receive (T*k of its own shard is
 * the usual figure), used only to choose the GEMM regime; t->hidden, t->out and
 * topk_* are unused. */
E4B_API size_t e4b_ep_experts_peer_workspace_bytes(const e4b_ep_peer_desc* pd, const e4b_moe_desc* local);
E4B_API e4b_status e4b_ep_experts_peer(const e4b_ep_peer_desc* pd, const e4b_moe_desc* local,
                               const e4b_moe_tensors* t, void* workspace, size_t workspace_bytes, void* stream);
E4B_API e4b_status e4b_ep_combine_peer(const e4b_ep_peer_desc* pd, const int32_t* inv, const void* topk_w,
                               int w_dtype, int T, int k, void* out, int out_dtype, void* stream);

/* ---- Resident / streamed expert stacks ----------------------------------
 * Replaces the address-table gather of the pipelined residency engine
 * (experts4bit_qlora/engines/pipelined.py:117-150, `_gather_rows_addr`, and the
 * resident-row dispatch of :300-340). Every expert's weights form one row-block of
 * four segments (gate_up packed, gate_up absmax, down packed, down absmax) at
 * seg_off_host[s] bytes, seg_bytes_host[s] long (both multiples of 16).
 * src_table [num_experts] (device) holds each row-block's address: device memory,
 * or pinned host memory (unified addressing). The fused layer reads four device
 * stacks seg_dst_host[s] = [resident_rows + slots, seg_bytes_host[s]]: rows
 * [0, resident_rows) hold resident experts, the rest one slot per pick. For pick
 * j < slots (ids [slots], device int64): if resident_row[ids[j]] >= 0 (device int32
 * [num_experts], nullable) the pick reads that row in place; otherwise slot j
 * receives expert ids[j]'s segments unless have[j] == ids[j] already (device int64
 * [slots], nullable: then every slot is copied), and have[j] is updated. local_ids
 * [slots] (device int64, nullable) receives the stack row of every pick: the
 * top-k index to pass to e4b_moe_forward over the stacks. The launch geometry does
 * not depend on the ids, so a decode step built on it can be captured in a CUDA
 * graph. An id outside [0, num_experts) is reported in the workspace's error word. */
E4B_API e4b_status e4b_gather_expert_rows(const uint64_t* src_table, int num_experts, const int64_t* ids,
                                  int64_t* have, int slots, const int32_t* resident_row, int resident_rows,
                                  int64_t* local_ids, const uint64_t* seg_off_host, const uint64_t* seg_bytes_host,
                                  void* const* seg_dst_host, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* Self-test of the failure path (no counterpart in the reference): one kernel
 * waits, with the library's bounded wait, on an asynchronous copy that is never
 * issued; the wait runs out, the kernel records E4B_ERR_TIMEOUT in the
 * workspace's error word (read it with e4b_read_device_error) and returns. The
 * second word of the workspace is 0 (timed out) or 1. Takes a few milliseconds. */
E4B_API e4b_status e4b_selftest_wait_timeout(void* workspace, size_t workspace_bytes, void* stream);

/* Reads (and clears) the device error word of a workspace used by the calls
 * above. Synchronises `stream`; for debugging and tests, not the hot path. */
E4B_API e4b_status e4b_read_device_error(void* workspace, void* stream, int* error_out);

/* Asynchronous watch of that word, for hosts that surface device errors without a
 * sync per call: returns the value the previous watch of this (workspace,
 * host_word, event) triple copied, if `event` (a cudaEvent_t) has completed,
 * else 0; then queues a 4-byte copy of the word into `host_word` (pinned host
 * memory) on `stream` and records `event` behind it. Non-zero: an earlier call
 * recorded that error; read and clear it with e4b_read_device_error. Not for use
 * inside a stream capture. */
E4B_API int e4b_watch_device_error(void* workspace, int* host_word, void* event, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* E4B_H_ */
