"""Tensor-level wrappers over the C ABI (include/e4b.h).

Each function validates shapes on the host, takes device memory from torch,
and launches on torch's current stream without synchronising. These are the
calls the module classes and the tests use.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N


def _cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor (the fused path has no CPU implementation)")


# --------------------------------------------------------------------------- #
# NF4 codec
# --------------------------------------------------------------------------- #
def nf4_quantize(w: torch.Tensor, blocksize: int = 64):
    """Blockwise NF4 of ``w`` (any shape, numel % 64 == 0) -> (packed u8 [n/2], absmax f32 [n/64]).

    Runs the CUDA kernel for CUDA tensors and the library's host routine for CPU
    tensors; both produce the same bytes."""
    if blocksize != 64:
        raise ValueError("only blocksize 64 is built")
    w = w.detach().contiguous()
    if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        w = w.float()
    n = w.numel()
    if n % 64:
        raise ValueError(f"element count {n} is not a multiple of 64")
    packed = torch.empty(n // 2, dtype=torch.uint8, device=w.device)
    absmax = torch.empty(n // 64, dtype=torch.float32, device=w.device)
    L = N.lib()
    if w.is_cuda:
        N.check(L.e4b_nf4_quantize(w.data_ptr(), N.dtype_code(w.dtype), n, packed.data_ptr(), absmax.data_ptr(),
                                   N.stream_handle(w.device)), "e4b_nf4_quantize")
    else:
        N.check(L.e4b_nf4_quantize_host(w.data_ptr(), N.dtype_code(w.dtype), n, packed.data_ptr(),
                                        absmax.data_ptr()), "e4b_nf4_quantize_host")
    return packed, absmax


def nf4_dequantize(packed: torch.Tensor, absmax: torch.Tensor, shape, dtype=torch.bfloat16) -> torch.Tensor:
    """``dtype(code[q] * absmax)``, reshaped to ``shape``."""
    packed = packed.contiguous()
    absmax = absmax.contiguous().float()
    n = packed.numel() * 2
    out = torch.empty(n, dtype=dtype, device=packed.device)
    L = N.lib()
    if packed.is_cuda:
        N.check(L.e4b_nf4_dequantize(packed.data_ptr(), absmax.data_ptr(), n, out.data_ptr(), N.dtype_code(dtype),
                                     N.stream_handle(packed.device)), "e4b_nf4_dequantize")
    else:
        N.check(L.e4b_nf4_dequantize_host(packed.data_ptr(), absmax.data_ptr(), n, out.data_ptr(),
                                          N.dtype_code(dtype)), "e4b_nf4_dequantize_host")
    return out.view(*shape)


def fp8_block_dequantize(w_u8: torch.Tensor, scale: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """``e4b_fp8_block_dequantize``: e4m3 bytes ``[out, in]`` with fp32 tile multipliers
    ``[ceil(out/128), ceil(in/128)]`` -> ``dtype`` (formats/fp8_blocks.py:60-128)."""
    _cuda(w_u8, "w")
    w = w_u8.contiguous()
    if w.dtype != torch.uint8:
        w = w.view(torch.uint8)
    rows, cols = w.shape
    if tuple(scale.shape) != ((rows + 127) // 128, (cols + 127) // 128):
        raise ValueError(f"scale {tuple(scale.shape)} does not tile a [{rows}, {cols}] weight at 128")
    sc = scale.float().contiguous()
    out = torch.empty(rows, cols, dtype=dtype, device=w.device)
    N.check(N.lib().e4b_fp8_block_dequantize(w.data_ptr(), sc.data_ptr(), rows, cols, out.data_ptr(),
                                             N.dtype_code(dtype), N.stream_handle(w.device)),
            "e4b_fp8_block_dequantize")
    return out


# --------------------------------------------------------------------------- #
# Router, permutation, grouped GEMM, combine
# --------------------------------------------------------------------------- #
def router_topk(x: torch.Tensor, router_weight: torch.Tensor, k: int, kind: int = N.SOFTMAX_THEN_TOPK,
                norm_topk_prob: bool = False, return_logits: bool = False):
    """fp32 router logits of ``x [T,H]`` against ``router_weight [E,H]`` and the
    deterministic top-k. Returns ``(weights f32 [T,k], idx i64 [T,k])`` (+ logits)."""
    _cuda(x, "x")
    x = x.contiguous()
    wr = router_weight.contiguous()
    T, H = x.shape
    E = wr.shape[0]
    dev = x.device
    idx = torch.empty(T, k, dtype=torch.int64, device=dev)
    w = torch.empty(T, k, dtype=torch.float32, device=dev)
    logits = torch.empty(T, E, dtype=torch.float32, device=dev) if return_logits else None
    L = N.lib()
    nbytes = _ROUTER_WS.get((T, E))
    if nbytes is None:
        nbytes = _ROUTER_WS[(T, E)] = L.e4b_router_workspace_bytes(T, E)
    ws = N.workspaces.get(dev, nbytes, "router")
    N.check(L.e4b_router_topk(x.data_ptr(), N.dtype_code(x.dtype), wr.data_ptr(), N.dtype_code(wr.dtype), T, H, E, k,
                              kind, int(norm_topk_prob), N.ptr(logits), idx.data_ptr(), w.data_ptr(),
                              ws.data_ptr(), ws.numel(), N.stream_handle(dev)), "e4b_router_topk")
    return (w, idx, logits) if return_logits else (w, idx)


def permute(top_k_index: torch.Tensor, num_experts: int):
    """Device permutation: ``(order i32 [T*k], inv i32 [T*k], offsets i32 [E+1])``."""
    _cuda(top_k_index, "top_k_index")
    idx = top_k_index.contiguous().long()
    T, k = idx.shape
    dev = idx.device
    order = torch.empty(T * k, dtype=torch.int32, device=dev)
    inv = torch.empty(T * k, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    L = N.lib()
    ws = N.workspaces.get(dev, L.e4b_permute_workspace_bytes(T, k, num_experts), "permute")
    N.check(L.e4b_permute(idx.data_ptr(), T, k, num_experts, order.data_ptr(), inv.data_ptr(), offsets.data_ptr(),
                          ws.data_ptr(), ws.numel(), N.stream_handle(dev)), "e4b_permute")
    return order, inv, offsets


def grouped_nf4_gemm(a: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor, offsets: torch.Tensor,
                     a_rows: torch.Tensor | None = None, epilogue: int = N.EPI_NONE) -> torch.Tensor:
    """Grouped NF4 GEMM: ``packed [E,N,K/2]``, ``absmax [E,N,K/64]``, expert-sorted rows
    delimited by ``offsets [E+1]`` (int32). Returns ``[R, N]`` (``[R, N/2]`` for SwiGLU)."""
    _cuda(a, "a")
    a = a.contiguous()
    E, Nn, Kh = packed.shape
    K = Kh * 2
    R = int(a_rows.numel()) if a_rows is not None else a.shape[0]
    n_out = Nn // 2 if epilogue == N.EPI_SWIGLU else Nn
    out = torch.empty(R, n_out, dtype=a.dtype, device=a.device)
    L = N.lib()
    ws = N.workspaces.get(a.device, L.e4b_grouped_gemm_workspace_bytes(R, E, Nn, K), "gemm")
    offs = offsets.to(torch.int32).contiguous()
    rows = a_rows.to(torch.int32).contiguous() if a_rows is not None else None
    N.check(L.e4b_grouped_nf4_gemm(a.data_ptr(), N.dtype_code(a.dtype), N.ptr(rows), packed.contiguous().data_ptr(),
                                   absmax.contiguous().data_ptr(), offs.data_ptr(), E, R, Nn, K, epilogue,
                                   out.data_ptr(), ws.data_ptr(), ws.numel(), N.stream_handle(a.device)),
            "e4b_grouped_nf4_gemm")
    return out


def dgrad_eligible(n: int, k: int) -> bool:
    """Shapes ``e4b_grouped_nf4_dgrad`` takes: ``W [E, n, k]`` with n % 64 == 0 and k % 256 == 0."""
    return n % 64 == 0 and k % 256 == 0


def grouped_nf4_dgrad(dy: torch.Tensor, packed: torch.Tensor, absmax: torch.Tensor, offsets: torch.Tensor,
                      out_dtype=torch.float32) -> torch.Tensor:
    """Input gradient of a frozen grouped NF4 projection: ``dx[r] = dy[r] . W_e`` for the
    expert-sorted rows of expert e (``offsets [E+1]``), with ``packed [E,N,K/2]`` /
    ``absmax [E,N,K/64]`` decoded on the fly. ``dy [R, N]`` bf16/fp16; returns ``[R, K]``."""
    _cuda(dy, "dy")
    dy = dy.contiguous()
    E, Nn, Kh = packed.shape
    K = Kh * 2
    R = dy.shape[0]
    if dy.dim() != 2 or dy.shape[1] != Nn:
        raise ValueError(f"dy must be [R, {Nn}], got {tuple(dy.shape)}")
    out = torch.empty(R, K, dtype=out_dtype, device=dy.device)
    L = N.lib()
    ws = N.workspaces.get(dy.device, L.e4b_grouped_nf4_dgrad_workspace_bytes(R, E, Nn, K), "dgrad")
    offs = offsets.to(torch.int32).contiguous()
    N.check(L.e4b_grouped_nf4_dgrad(dy.data_ptr(), N.dtype_code(dy.dtype), packed.contiguous().data_ptr(),
                                    absmax.contiguous().data_ptr(), offs.data_ptr(), E, R, Nn, K, out.data_ptr(),
                                    N.dtype_code(out_dtype), ws.data_ptr(), ws.numel(), N.stream_handle(dy.device)),
            "e4b_grouped_nf4_dgrad")
    return out


def combine(rows: torch.Tensor, inv: torch.Tensor, w: torch.Tensor | None, tokens: int, k: int,
            out_dtype=torch.bfloat16) -> torch.Tensor:
    _cuda(rows, "rows")
    rows = rows.contiguous()
    H = rows.shape[1]
    out = torch.empty(tokens, H, dtype=out_dtype, device=rows.device)
    w = w.contiguous() if w is not None else None  # None: every weight 1 (the plain slot sum)
    N.check(N.lib().e4b_combine(rows.data_ptr(), N.dtype_code(rows.dtype), inv.to(torch.int32).contiguous().data_ptr(),
                                N.ptr(w), N.dtype_code(w.dtype) if w is not None else N.F32, tokens, k, H,
                                out.data_ptr(), N.dtype_code(out_dtype), N.stream_handle(rows.device)), "e4b_combine")
    return out


class RowTiles:
    """Expert-sorted rows as device tables for the adapter kernels: ``tiles`` [(expert, first row,
    rows <= 32)] and ``segs`` [(expert, first row, rows)] of the experts with rows, built from the
    host copy of the offsets [E+1]."""

    def __init__(self, offsets_host, device):
        import numpy as np
        off = np.asarray(offsets_host, dtype=np.int64)
        cnt = off[1:] - off[:-1]
        act = np.nonzero(cnt > 0)[0]
        ntile = (cnt[act] + 31) // 32
        e_t = np.repeat(act, ntile)
        first = np.repeat(np.cumsum(ntile) - ntile, ntile)
        j = np.arange(int(ntile.sum())) - first
        row0 = off[e_t] + 32 * j
        rows = np.minimum(32, off[e_t + 1] - row0)
        self.ntiles, self.nsegs = int(len(e_t)), int(len(act))
        tiles = np.stack([e_t, row0, rows], 1).astype(np.int32).reshape(-1)
        segs = np.stack([act, off[act], cnt[act]], 1).astype(np.int32).reshape(-1)
        both = torch.from_numpy(np.concatenate([tiles, segs])).pin_memory()
        dev = both.to(device, non_blocking=True)
        self.tiles, self.segs = dev[:tiles.size], dev[tiles.size:]
        self._host = both  # kept until the copy has run


def lora_rank_down(X: torch.Tensor, M: torch.Tensor, strides, rk: int, tiles: RowTiles,
                   scale: float = 1.0) -> torch.Tensor:
    """``Y [R, rk] = scale * X[row] . M_e(j, :)`` over expert-sorted rows (fp32, ranks <= 16);
    ``strides = (sE, sj, sk)`` address ``M_e(j, k)`` in the fp32 tensor ``M``."""
    X = X.contiguous()
    M = M.float().contiguous()
    R, K = X.shape
    Y = torch.empty(R, rk, dtype=torch.float32, device=X.device)
    N.check(N.lib().e4b_lora_rank_down(X.data_ptr(), N.dtype_code(X.dtype), K, M.data_ptr(), *strides, rk, K,
                                       tiles.tiles.data_ptr(), tiles.ntiles, float(scale), Y.data_ptr(),
                                       N.stream_handle(X.device)), "e4b_lora_rank_down")
    return Y


def lora_rank_up(Y: torch.Tensor, M: torch.Tensor, strides, n: int, tiles: RowTiles, out: torch.Tensor,
                 scale: float = 1.0) -> torch.Tensor:
    """``out[row, :n] += scale * Y[row] . M_e(:, n)`` in place: fp32 ``out`` accumulates; a 16-bit
    ``out`` gets the delta rounded to its dtype first (as a 16-bit projection plus its delta)."""
    M = M.float().contiguous()
    rk = Y.shape[1]
    mode = 1 if out.dtype == torch.float32 else 2
    N.check(N.lib().e4b_lora_rank_up(Y.data_ptr(), rk, M.data_ptr(), *strides, n, tiles.tiles.data_ptr(),
                                     tiles.ntiles, float(scale), mode, out.data_ptr(), N.dtype_code(out.dtype),
                                     out.shape[1], N.stream_handle(Y.device)), "e4b_lora_rank_up")
    return out


def lora_outer(P: torch.Tensor, Y: torch.Tensor, tiles: RowTiles, G: torch.Tensor, strides,
               scale: float = 1.0) -> torch.Tensor:
    """``G_e(a, j) = scale * sum over the rows of e of P[row, a] * Y[row, j]`` into the fp32 tensor
    ``G`` (``strides = (gE, ga, gj)``); experts without rows are left as they are."""
    P = P.contiguous()
    A = P.shape[1]
    N.check(N.lib().e4b_lora_outer(P.data_ptr(), N.dtype_code(P.dtype), A, A, Y.data_ptr(), Y.shape[1],
                                   tiles.segs.data_ptr(), tiles.nsegs, float(scale), G.data_ptr(), *strides,
                                   N.stream_handle(P.device)), "e4b_lora_outer")
    return G


def swiglu_forward(proj: torch.Tensor, has_gate: bool = True) -> torch.Tensor:
    """``act(gate) * up`` of expert-sorted projection rows ``[R, 2I]`` (or ``act(proj)``)."""
    _cuda(proj, "proj")
    proj = proj.contiguous()
    R, n1 = proj.shape
    I = n1 // 2 if has_gate else n1
    h = torch.empty(R, I, dtype=proj.dtype, device=proj.device)
    N.check(N.lib().e4b_swiglu_forward(proj.data_ptr(), N.dtype_code(proj.dtype), R, I, int(has_gate), h.data_ptr(),
                                       N.stream_handle(proj.device)), "e4b_swiglu_forward")
    return h


def swiglu_backward(proj: torch.Tensor, dh: torch.Tensor, has_gate: bool = True) -> torch.Tensor:
    """dL/d(proj) in proj's dtype from dL/dh (fp32 ``[R, I]``)."""
    _cuda(proj, "proj")
    proj = proj.contiguous()
    dh = dh.float().contiguous()
    R, n1 = proj.shape
    I = n1 // 2 if has_gate else n1
    if tuple(dh.shape) != (R, I):
        raise ValueError(f"dh must be [{R}, {I}], got {tuple(dh.shape)}")
    dproj = torch.empty_like(proj)
    N.check(N.lib().e4b_swiglu_backward(proj.data_ptr(), N.dtype_code(proj.dtype), dh.data_ptr(), R, I, int(has_gate),
                                        dproj.data_ptr(), N.stream_handle(proj.device)), "e4b_swiglu_backward")
    return dproj


def combine_row_grads(grad: torch.Tensor, token_rows: torch.Tensor, w_rows: torch.Tensor, down: torch.Tensor):
    """Gradients of ``out[t] = sum_s w down[row]`` per expert-sorted row: ``(dd [R, H] in down's dtype,
    dw fp32 [R])`` from dL/dout (fp32 ``[T, H]``)."""
    _cuda(grad, "grad")
    grad = grad.float().contiguous()
    down = down.contiguous()
    rows = token_rows.long().contiguous()
    w = w_rows.float().contiguous()
    R, H = down.shape
    if grad.shape[1] != H or rows.numel() != R or w.numel() != R:
        raise ValueError("combine_row_grads: grad [T, H], token_rows [R], w_rows [R], down [R, H]")
    dd = torch.empty_like(down)
    dw = torch.empty(R, dtype=torch.float32, device=down.device)
    N.check(N.lib().e4b_combine_row_grads(grad.data_ptr(), rows.data_ptr(), w.data_ptr(), down.data_ptr(),
                                          N.dtype_code(down.dtype), R, H, dd.data_ptr(), dw.data_ptr(),
                                          N.stream_handle(down.device)), "e4b_combine_row_grads")
    return dd, dw


# --------------------------------------------------------------------------- #
# Whole layer
# --------------------------------------------------------------------------- #
def _expect(t: torch.Tensor, what: str, device, dtypes, numel: int | None = None, shape=None) -> None:
    """Raise ValueError unless ``t`` is a contiguous tensor on ``device`` with one of ``dtypes`` and the
    given element count / shape: the kernels read raw pointers, so a mismatch would read out of bounds."""
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{what} must be a tensor")
    if t.device != device:
        raise ValueError(f"{what} is on {t.device}, expected {device}")
    if t.dtype not in dtypes:
        raise ValueError(f"{what} has dtype {t.dtype}, expected one of {tuple(dtypes)}")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{what} has {t.numel()} elements, expected {numel}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{what} has shape {tuple(t.shape)}, expected {tuple(shape)}")


_VALIDATED: dict = {}  # stacks already checked for this geometry (bounded; keys hold no tensors)
_DESCS: dict = {}  # layer descriptor per call signature (bounded)
_ROUTER_WS: dict = {}  # router workspace size per (T, E)


def _check_layer(dev, E, H, I, has_gate, gate_up_packed, gate_up_absmax, down_packed, down_absmax, weight_format,
                 lora=None):
    key = None
    if lora is None:
        key = (dev, E, H, I, has_gate, weight_format) + tuple(
            (m.data_ptr(), m.numel(), m.dtype, m.device) for m in (gate_up_packed, gate_up_absmax, down_packed,
                                                                   down_absmax))
        if key in _VALIDATED:
            return
    _check_layer_full(dev, E, H, I, has_gate, gate_up_packed, gate_up_absmax, down_packed, down_absmax,
                      weight_format, lora)
    if key is not None:
        if len(_VALIDATED) > 4096:
            _VALIDATED.clear()
        _VALIDATED[key] = True


def _check_layer_full(dev, E, H, I, has_gate, gate_up_packed, gate_up_absmax, down_packed, down_absmax,
                      weight_format, lora=None):
    n1 = 2 * I if has_gate else I
    if weight_format == N.FMT_MXFP4:
        _expect(gate_up_packed, "gate_up codes", dev, (torch.uint8,), E * n1 * H // 2)
        _expect(down_packed, "down codes", dev, (torch.uint8,), E * H * I // 2)
        _expect(gate_up_absmax, "gate_up e8m0 scales", dev, (torch.uint8,), E * n1 * H // 32)
        _expect(down_absmax, "down e8m0 scales", dev, (torch.uint8,), E * H * I // 32)
    elif weight_format == N.FMT_FP8_BLOCK128:
        _expect(gate_up_packed, "gate_up weights", dev, (torch.uint8,), E * n1 * H)
        _expect(down_packed, "down weights", dev, (torch.uint8,), E * H * I)
        _expect(gate_up_absmax, "gate_up scales", dev, (torch.float32,), E * (n1 // 128) * (H // 128))
        _expect(down_absmax, "down scales", dev, (torch.float32,), E * (H // 128) * (I // 128))
    else:
        _expect(gate_up_packed, "gate_up_proj", dev, (torch.uint8,), E * n1 * H // 2)
        _expect(down_packed, "down_proj", dev, (torch.uint8,), E * H * I // 2)
        _expect(gate_up_absmax, "gate_up_absmax", dev, (torch.float32,), E * n1 * H // 64)
        _expect(down_absmax, "down_absmax", dev, (torch.float32,), E * H * I // 64)
    if lora is not None:
        A_gu, B_gu, A_dn, B_dn = lora[:4]
        if A_gu.dim() != 3:
            raise ValueError("LoRA A of gate_up must be [E, r, H]")
        r = A_gu.shape[1]
        dts = (A_gu.dtype,)
        if A_gu.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError(f"LoRA dtype {A_gu.dtype} is not bf16/fp16/fp32")
        for m, what, shape in ((A_gu, "gate_up LoRA A", (E, r, H)), (B_gu, "gate_up LoRA B", (E, n1, r)),
                               (A_dn, "down LoRA A", (E, r, I)), (B_dn, "down LoRA B", (E, H, r))):
            if m.device != dev or m.dtype not in dts or tuple(m.shape) != shape:
                raise ValueError(f"{what}: expected {shape} {A_gu.dtype} on {dev}, got {tuple(m.shape)} "
                                 f"{m.dtype} on {m.device}")


def moe_forward(hidden: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                gate_up_packed: torch.Tensor, gate_up_absmax: torch.Tensor, down_packed: torch.Tensor,
                down_absmax: torch.Tensor, num_experts: int, intermediate: int, has_gate: bool = True,
                out_dtype=None, lora=None, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                check_errors: bool = False, weight_format: int = N.FMT_NF4,
                expert_map: torch.Tensor | None = None) -> torch.Tensor:
    """One fused expert layer through ``e4b_moe_forward``.

    ``hidden [T,H]`` must already be in the compute dtype (bf16/fp16).
    ``lora`` = ``(A_gu [E,r,H], B_gu [E,n1,r], A_dn [E,r,I], B_dn [E,H,r], scaling)`` or None.
    ``weight_format`` = ``FMT_FP8_BLOCK128``: the ``*_packed`` stacks are e4m3 bytes and the
    ``*_absmax`` stacks fp32 tile multipliers (bf16 activations, no adapters).
    ``expert_map`` (int32 ``[routed]``): the stacks hold a sub-stack of ``num_experts`` resident
    experts; the top-k ids lie in ``[0, routed)`` and ``expert_map[id]`` is the expert's index in
    the stacks (-1 = not resident, a device error).
    """
    _cuda(hidden, "hidden_states")
    if hidden.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError("hidden must be bf16 or fp16 (the compute dtype)")
    hidden = hidden.contiguous()
    idx = top_k_index.contiguous()
    if idx.dtype != torch.int64:
        idx = idx.long()
    w = top_k_weights.contiguous()
    if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        w = w.float()
    if hidden.dim() != 2 or idx.dim() != 2 or idx.shape[0] != hidden.shape[0]:
        raise ValueError(f"hidden {tuple(hidden.shape)} and top_k_index {tuple(idx.shape)} must be [T, H] and [T, k]")
    T, H = hidden.shape
    k = idx.shape[1]
    dev = hidden.device
    _expect(idx, "top_k_index", dev, (torch.int64,), shape=(T, k))
    _expect(w, "top_k_weights", dev, (torch.bfloat16, torch.float16, torch.float32), shape=(T, k))
    _check_layer(dev, num_experts, H, intermediate, has_gate, gate_up_packed, gate_up_absmax, down_packed,
                 down_absmax, weight_format, lora)
    out_dtype = out_dtype or hidden.dtype
    if out is None:
        out = torch.empty(T, H, dtype=out_dtype, device=hidden.device)
    _expect(out, "out", dev, (out_dtype,), shape=(T, H))
    routed = int(expert_map.numel()) if expert_map is not None else 0
    sig = (num_experts, H, intermediate, k, T, bool(has_gate), hidden.dtype, w.dtype, out_dtype, weight_format,
           routed, None if lora is None else (lora[0].shape[1], lora[0].dtype, float(lora[4])))
    d = _DESCS.get(sig)  # the descriptor is only read by the library
    if d is None:
        d = MoeDesc_from(num_experts, H, intermediate, k, T, has_gate, hidden.dtype, w.dtype, out_dtype, lora,
                         weight_format)
        d.routed_experts = routed
        if len(_DESCS) > 4096:
            _DESCS.clear()
        _DESCS[sig] = d
    t = N.MoeTensors()
    t.hidden, t.topk_idx, t.topk_w = hidden.data_ptr(), idx.data_ptr(), w.data_ptr()
    t.gate_up_packed, t.gate_up_absmax = gate_up_packed.data_ptr(), gate_up_absmax.data_ptr()
    t.down_packed, t.down_absmax = down_packed.data_ptr(), down_absmax.data_ptr()
    keep = []
    if lora is not None:
        A_gu, B_gu, A_dn, B_dn, _ = lora
        mats = [m.contiguous() for m in (A_gu, B_gu, A_dn, B_dn)]
        keep = mats
        t.gate_up_lora_A, t.gate_up_lora_B, t.down_lora_A, t.down_lora_B = (m.data_ptr() for m in mats)
    t.out = out.data_ptr()
    if expert_map is not None:
        _expect(expert_map, "expert_map", dev, (torch.int32,))
        t.expert_map = expert_map.data_ptr()
    L = N.lib()
    nbytes = L.e4b_moe_workspace_bytes(ctypes.byref(d))  # depends on the decode-kernel selection too
    if nbytes == 0:
        raise ValueError("invalid expert-layer geometry for the fused kernel")
    ws = workspace if workspace is not None else N.workspaces.get(hidden.device, nbytes, "moe")
    if ws.numel() < nbytes:
        raise ValueError(f"workspace of {ws.numel()} bytes < required {nbytes}")
    N.check(L.e4b_moe_forward(ctypes.byref(d), ctypes.byref(t), ws.data_ptr(), ws.numel(),
                              N.stream_handle(hidden.device)), "e4b_moe_forward")
    del keep
    if check_errors:
        err = N.read_device_error(ws)
        if err:
            raise N.E4BError(err, "e4b_moe_forward (device)")
    else:
        N.error_watch.after(ws, "e4b_moe_forward")
    return out


def moe_decode_step(hidden: torch.Tensor, router_weight: torch.Tensor, top_k: int, gate_up_packed: torch.Tensor,
                    gate_up_absmax: torch.Tensor, down_packed: torch.Tensor, down_absmax: torch.Tensor,
                    num_experts: int, intermediate: int, has_gate: bool = True, kind: int = N.SOFTMAX_THEN_TOPK,
                    norm_topk_prob: bool = False, out_dtype=None, out: torch.Tensor | None = None,
                    topk_idx: torch.Tensor | None = None, topk_w: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None, check_errors: bool = False, stage_events=None):
    """Router and expert layer in one call (``e4b_moe_decode_step``): top-k of the fp32 logits
    ``hidden . router_weight^T``, then the fused layer with those picks. In the decode regime
    both run in a single launch. Returns ``(out [T,H], top_k_weights f32 [T,k], top_k_index i64 [T,k])``."""
    _cuda(hidden, "hidden_states")
    hidden = hidden.contiguous()
    T, H = hidden.shape
    dev = hidden.device
    out_dtype = out_dtype or hidden.dtype
    out = out if out is not None else torch.empty(T, H, dtype=out_dtype, device=dev)
    topk_idx = topk_idx if topk_idx is not None else torch.empty(T, top_k, dtype=torch.int64, device=dev)
    topk_w = topk_w if topk_w is not None else torch.empty(T, top_k, dtype=torch.float32, device=dev)
    wr = router_weight.contiguous()
    _expect(wr, "router_weight", dev, (torch.bfloat16, torch.float16, torch.float32), shape=(num_experts, H))
    _expect(out, "out", dev, (out_dtype,), shape=(T, H))
    _expect(topk_idx, "topk_idx", dev, (torch.int64,), shape=(T, top_k))
    _expect(topk_w, "topk_w", dev, (torch.float32,), shape=(T, top_k))
    _check_layer(dev, num_experts, H, intermediate, has_gate, gate_up_packed, gate_up_absmax, down_packed,
                 down_absmax, N.FMT_NF4)
    d = MoeDesc_from(num_experts, H, intermediate, top_k, T, has_gate, hidden.dtype, torch.float32, out_dtype, None)
    t = N.MoeTensors()
    t.hidden = hidden.data_ptr()
    t.gate_up_packed, t.gate_up_absmax = gate_up_packed.data_ptr(), gate_up_absmax.data_ptr()
    t.down_packed, t.down_absmax = down_packed.data_ptr(), down_absmax.data_ptr()
    t.out = out.data_ptr()
    keep = None
    if stage_events is not None:
        keep = (ctypes.c_void_p * N.MOE_STAGE_EVENTS)(*stage_events)
        t.stage_events = ctypes.cast(keep, ctypes.c_void_p)
    L = N.lib()
    nbytes = L.e4b_moe_decode_step_workspace_bytes(ctypes.byref(d))
    if nbytes == 0:
        raise ValueError("invalid expert-layer geometry for the fused kernel")
    ws = workspace if workspace is not None else N.workspaces.get(dev, nbytes, "moe_step")
    if ws.numel() < nbytes:
        raise ValueError(f"workspace of {ws.numel()} bytes < required {nbytes}")
    N.check(L.e4b_moe_decode_step(ctypes.byref(d), ctypes.byref(t), wr.data_ptr(), N.dtype_code(wr.dtype), kind,
                                  int(norm_topk_prob), topk_idx.data_ptr(), topk_w.data_ptr(), ws.data_ptr(),
                                  ws.numel(), N.stream_handle(dev)), "e4b_moe_decode_step")
    del keep
    if check_errors:
        err = N.read_device_error(ws)
        if err:
            raise N.E4BError(err, "e4b_moe_decode_step (device)")
    else:
        N.error_watch.after(ws, "e4b_moe_decode_step")
    return out, topk_w, topk_idx


def MoeDesc_from(E, H, I, k, T, has_gate, act_dtype, w_dtype, out_dtype, lora, weight_format=N.FMT_NF4) -> N.MoeDesc:
    d = N.MoeDesc()
    d.weight_format = int(weight_format)
    d.num_experts, d.hidden, d.intermediate, d.top_k, d.tokens = E, H, I, k, T
    d.has_gate = int(bool(has_gate))
    d.act_dtype = N.dtype_code(act_dtype)
    d.weight_dtype = N.dtype_code(w_dtype)
    d.out_dtype = N.dtype_code(out_dtype)
    if lora is not None:
        A_gu = lora[0]
        d.lora_rank = A_gu.shape[1]
        d.lora_dtype = N.dtype_code(A_gu.dtype)
        d.lora_scaling = float(lora[4])
    return d


def moe_path(E, H, I, k, T, has_gate=True, act_dtype=torch.bfloat16, lora_rank=0, weight_format=N.FMT_NF4) -> int:
    """Which kernel sequence ``e4b_moe_forward`` runs (``_native.PATH_*``)."""
    d = N.MoeDesc()
    d.num_experts, d.hidden, d.intermediate, d.top_k, d.tokens = E, H, I, k, T
    d.has_gate = int(bool(has_gate))
    d.act_dtype = N.dtype_code(act_dtype)
    d.weight_dtype = N.F32
    d.out_dtype = N.dtype_code(act_dtype)
    d.lora_rank = lora_rank
    d.lora_dtype = N.F32
    d.weight_format = int(weight_format)
    return N.lib().e4b_moe_path(ctypes.byref(d))


def moe_decode_step_workspace_bytes(E, H, I, k, T, has_gate=True, act_dtype=torch.bfloat16) -> int:
    d = MoeDesc_from(E, H, I, k, T, has_gate, act_dtype, torch.float32, act_dtype, None)
    return N.lib().e4b_moe_decode_step_workspace_bytes(ctypes.byref(d))


def set_decode_kernel(mode) -> int:
    """Select the one-launch decode-layer kernel for the process; returns the old setting.

    ``False``/0 turns it off, 1 selects the flow kernel where it applies, 2 the phase kernel,
    ``True``/3 the slice kernel where it applies (the default)."""
    m = 3 if mode is True else 0 if mode is False else int(mode)
    return N.lib().e4b_set_decode_kernel(m)


def moe_workspace_bytes(E, H, I, k, T, has_gate=True, act_dtype=torch.bfloat16, lora_rank=0,
                        weight_format=N.FMT_NF4) -> int:
    d = N.MoeDesc()
    d.weight_format = int(weight_format)
    d.num_experts, d.hidden, d.intermediate, d.top_k, d.tokens = E, H, I, k, T
    d.has_gate = int(bool(has_gate))
    d.act_dtype = N.dtype_code(act_dtype)
    d.weight_dtype = N.F32
    d.out_dtype = N.dtype_code(act_dtype)
    d.lora_rank = lora_rank
    d.lora_dtype = N.F32
    return N.lib().e4b_moe_workspace_bytes(ctypes.byref(d))
