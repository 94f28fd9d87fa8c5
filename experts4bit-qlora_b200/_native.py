"""ctypes binding of libe4b.so (the C ABI declared in include/e4b.h).

The fused path has no CPU fallback: if the library is missing, every call
raises ``NativeLibraryError``. torch is used only for device memory and the
current CUDA stream.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libe4b.so")

E4B_OK = 0
E4B_ERR_EXPERT_INDEX = 6
E4B_ERR_RANGE = 7
E4B_ERR_TIMEOUT = 8
BF16, F16, F32 = 0, 1, 2
SOFTMAX_THEN_TOPK, TOPK_THEN_SOFTMAX = 0, 1
EPI_NONE, EPI_SWIGLU, EPI_SILU = 0, 1, 2
FMT_NF4, FMT_FP8_BLOCK128, FMT_MXFP4 = 0, 1, 2
PATH_STREAMING, PATH_TENSOR_CORE, PATH_DECODE_LAYER = 0, 1, 2
ABI_VERSION = 4

# Every symbol include/e4b.h exports, in declaration order.
EXPORTED_SYMBOLS = (
    "e4b_status_string", "e4b_abi_version",
    "e4b_nf4_quantize", "e4b_nf4_dequantize", "e4b_nf4_quantize_host", "e4b_nf4_dequantize_host",
    "e4b_router_workspace_bytes", "e4b_router_topk",
    "e4b_permute_workspace_bytes", "e4b_permute",
    "e4b_fp8_block_dequantize",
    "e4b_mxfp4_dequantize", "e4b_mxfp4_dequantize_host",
    "e4b_grouped_gemm_workspace_bytes", "e4b_grouped_nf4_gemm",
    "e4b_grouped_nf4_dgrad_workspace_bytes", "e4b_grouped_nf4_dgrad",
    "e4b_combine",
    "e4b_swiglu_forward", "e4b_swiglu_backward", "e4b_combine_row_grads",
    "e4b_lora_rank_down", "e4b_lora_rank_up", "e4b_lora_outer",
    "e4b_moe_workspace_bytes", "e4b_moe_forward",
    "e4b_moe_decode_step_workspace_bytes", "e4b_moe_decode_step",
    "e4b_moe_path", "e4b_set_decode_kernel",
    "e4b_moe_forward_static",
    "e4b_ep_dispatch_workspace_bytes", "e4b_ep_dispatch", "e4b_ep_experts_workspace_bytes", "e4b_ep_experts",
    "e4b_ep_comm_bytes", "e4b_ipc_export", "e4b_ipc_open", "e4b_ipc_close",
    "e4b_ep_dispatch_peer_workspace_bytes", "e4b_ep_dispatch_peer",
    "e4b_ep_experts_peer_workspace_bytes", "e4b_ep_experts_peer", "e4b_ep_combine_peer",
    "e4b_gather_expert_rows",
    "e4b_selftest_wait_timeout",
    "e4b_read_device_error", "e4b_watch_device_error",
)


class NativeLibraryError(RuntimeError):
    """libe4b.so is missing or failed to load: the fused path cannot run."""


class E4BError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


class MoeDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "num_experts", "hidden", "intermediate", "top_k", "tokens", "has_gate", "act_dtype",
        "weight_dtype", "out_dtype", "lora_rank", "lora_dtype")] + [("lora_scaling", ctypes.c_float),
                                                                     ("weight_format", ctypes.c_int),
                                                                     ("routed_experts", ctypes.c_int)]


class MoeTensors(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "hidden", "topk_idx", "topk_w", "gate_up_packed", "gate_up_absmax", "down_packed", "down_absmax",
        "gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B", "out", "stage_events", "expert_map")]

MOE_STAGE_EVENTS = 7
IPC_HANDLE_BYTES = 64
EP_MAX_PEERS = 16


class EpPeerDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("world", "rank", "local_experts", "rows_per_rank", "hidden",
                                            "act_dtype")] + [("peers", ctypes.c_void_p)]


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P, I, SZ, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_int64, ctypes.c_float
    sig = {
        "e4b_status_string": (ctypes.c_char_p, [I]),
        "e4b_abi_version": (I, []),
        "e4b_nf4_quantize": (I, [P, I, I64, P, P, P]),
        "e4b_nf4_dequantize": (I, [P, P, I64, P, I, P]),
        "e4b_nf4_quantize_host": (I, [P, I, I64, P, P]),
        "e4b_nf4_dequantize_host": (I, [P, P, I64, P, I]),
        "e4b_router_workspace_bytes": (SZ, [I, I]),
        "e4b_router_topk": (I, [P, I, P, I, I, I, I, I, I, I, P, P, P, P, SZ, P]),
        "e4b_permute_workspace_bytes": (SZ, [I, I, I]),
        "e4b_permute": (I, [P, I, I, I, P, P, P, P, SZ, P]),
        "e4b_fp8_block_dequantize": (I, [P, P, I64, I64, P, I, P]),
        "e4b_mxfp4_dequantize": (I, [P, P, I64, I64, I64, I64, P, I, P]),
        "e4b_mxfp4_dequantize_host": (I, [P, P, I64, I64, I64, I64, P, I]),
        "e4b_grouped_gemm_workspace_bytes": (SZ, [I, I, I, I]),
        "e4b_grouped_nf4_gemm": (I, [P, I, P, P, P, P, I, I, I, I, I, P, P, SZ, P]),
        "e4b_grouped_nf4_dgrad_workspace_bytes": (SZ, [I, I, I, I]),
        "e4b_grouped_nf4_dgrad": (I, [P, I, P, P, P, I, I, I, I, P, I, P, SZ, P]),
        "e4b_combine": (I, [P, I, P, P, I, I, I, I, P, I, P]),
        "e4b_swiglu_forward": (I, [P, I, ctypes.c_int64, I, I, P, P]),
        "e4b_swiglu_backward": (I, [P, I, P, ctypes.c_int64, I, I, P, P]),
        "e4b_combine_row_grads": (I, [P, P, P, P, I, ctypes.c_int64, I, P, P, P]),
        "e4b_lora_rank_down": (I, [P, I, I, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, I, I, P, I,
                                   ctypes.c_float, P, P]),
        "e4b_lora_rank_up": (I, [P, I, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, I, P, I, ctypes.c_float, I,
                                 P, I, I, P]),
        "e4b_lora_outer": (I, [P, I, I, I, P, I, P, I, ctypes.c_float, P, ctypes.c_int64, ctypes.c_int64,
                               ctypes.c_int64, P]),
        "e4b_moe_workspace_bytes": (SZ, [ctypes.POINTER(MoeDesc)]),
        "e4b_moe_forward": (I, [ctypes.POINTER(MoeDesc), ctypes.POINTER(MoeTensors), P, SZ, P]),
        "e4b_moe_forward_static": (I, [ctypes.POINTER(MoeDesc), ctypes.POINTER(MoeTensors), P]),
        "e4b_moe_path": (I, [ctypes.POINTER(MoeDesc)]),
        "e4b_moe_decode_step_workspace_bytes": (SZ, [ctypes.POINTER(MoeDesc)]),
        "e4b_moe_decode_step": (I, [ctypes.POINTER(MoeDesc), ctypes.POINTER(MoeTensors), P, I, I, I, P, P, P, SZ, P]),
        "e4b_set_decode_kernel": (I, [I]),
        "e4b_ep_dispatch_workspace_bytes": (SZ, [I, I, I]),
        "e4b_ep_dispatch": (I, [P, I, P, I, I, I, I, P, P, P, P, SZ, P]),
        "e4b_ep_experts_workspace_bytes": (SZ, [ctypes.POINTER(MoeDesc), I]),
        "e4b_ep_experts": (I, [ctypes.POINTER(MoeDesc), I, P, ctypes.POINTER(MoeTensors), P, SZ, P]),
        "e4b_ep_comm_bytes": (SZ, [I, I, I, I]),
        "e4b_ipc_export": (I, [P, P, ctypes.POINTER(SZ)]),
        "e4b_ipc_open": (I, [P, SZ, ctypes.POINTER(P)]),
        "e4b_ipc_close": (I, [P, SZ]),
        "e4b_ep_dispatch_peer_workspace_bytes": (SZ, [I, I, I]),
        "e4b_ep_dispatch_peer": (I, [ctypes.POINTER(EpPeerDesc), P, P, I, I, P, P, SZ, P]),
        "e4b_ep_experts_peer_workspace_bytes": (SZ, [ctypes.POINTER(EpPeerDesc), ctypes.POINTER(MoeDesc)]),
        "e4b_ep_experts_peer": (I, [ctypes.POINTER(EpPeerDesc), ctypes.POINTER(MoeDesc), ctypes.POINTER(MoeTensors),
                                    P, SZ, P]),
        "e4b_ep_combine_peer": (I, [ctypes.POINTER(EpPeerDesc), P, P, I, I, I, P, I, P]),
        "e4b_gather_expert_rows": (I, [P, I, P, P, I, P, I, P, P, P, P, P, SZ, P]),
        "e4b_selftest_wait_timeout": (I, [P, SZ, P]),
        "e4b_read_device_error": (I, [P, P, ctypes.POINTER(I)]),
        "e4b_watch_device_error": (I, [P, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del F


def lib():
    """The loaded library; raises NativeLibraryError when it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise NativeLibraryError(
                        f"{LIB_PATH} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                        "(or experts4bit-qlora_b200/build.py). There is no CPU fallback for the fused path.")
                try:
                    l = ctypes.CDLL(LIB_PATH)
                except OSError as e:
                    raise NativeLibraryError(f"failed to load {LIB_PATH}: {e}") from e
                _declare(l)
                if l.e4b_abi_version() != ABI_VERSION:
                    raise NativeLibraryError("libe4b.so ABI version mismatch; rebuild it")
                _lib = l
    return _lib


def available() -> bool:
    try:
        lib()
        return True
    except NativeLibraryError:
        return False


def status_string(status: int) -> str:
    try:
        return lib().e4b_status_string(int(status)).decode()
    except NativeLibraryError:
        return "native library unavailable"


def check(status: int, what: str) -> None:
    if status != E4B_OK:
        raise E4BError(status, what)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    if dt == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {dt}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The raw cudaStream_t of torch's current stream on ``device`` (a hot-path call: torch's
    private raw-stream query when present, which skips building a Stream object)."""
    if _raw_stream is not None:
        idx = device.index if isinstance(device, torch.device) else device
        return _raw_stream(idx if idx is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


class _Workspaces:
    """One grow-only workspace per (device, purpose), owned by torch's allocator.

    Reusing a buffer keeps its address stable across calls, which CUDA-graph
    replay needs. Calls on one device that share a purpose must be
    stream-ordered (the library is stream-ordered; this cache is not a pool).

    Buffers start zero-filled: the library's workspace header (the sticky
    error word and the decode kernel's counter block) must be zero before its
    first use, and the library leaves it that way. A buffer that is outgrown
    is kept alive, not freed: a CUDA graph captured before the growth still
    writes to it on every replay.
    """

    def __init__(self):
        self._bufs: dict[tuple[int, str], torch.Tensor] = {}
        self._retired: list[torch.Tensor] = []
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int, purpose: str = "moe") -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), purpose)
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                if buf is not None:
                    self._retired.append(buf)
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                self._bufs[key] = buf
            return buf


workspaces = _Workspaces()


def read_device_error(ws: torch.Tensor) -> int:
    out = ctypes.c_int(0)
    check(lib().e4b_read_device_error(ws.data_ptr(), stream_handle(ws.device), ctypes.byref(out)),
          "e4b_read_device_error")
    return out.value


class _ErrorWatch:
    """Surfaces the sticky device error word of a workspace without a per-call host sync.

    After a call, one library call (``e4b_watch_device_error``) queues a 4-byte copy of the
    word into pinned host memory behind an event and returns what the previous copy found
    once its event has completed; a non-zero value is read and cleared (one sync, only then)
    and raised. ``check_errors()`` synchronises and raises at once. Calls inside a CUDA-graph
    capture are not watched (a capture cannot record host reads).
    """

    def __init__(self):
        self._w: dict[int, tuple[torch.Tensor, torch.Tensor, object]] = {}
        self._lock = threading.Lock()

    def before(self, ws: torch.Tensor, what: str) -> None:
        """Kept for callers that check before a launch: the watch itself runs in ``after``."""

    def after(self, ws: torch.Tensor, what: str = "call") -> None:
        ent = self._w.get(ws.data_ptr())
        if ent is None:
            if torch.cuda.is_current_stream_capturing():
                return
            with self._lock:
                ent = self._w.get(ws.data_ptr())
                if ent is None:
                    ev = torch.cuda.Event()
                    ev.record()  # torch creates the CUDA event on its first record
                    ent = (torch.zeros(1, dtype=torch.int32, pin_memory=True), ws, ev)
                    self._w[ws.data_ptr()] = ent
        elif torch.cuda.is_current_stream_capturing():
            return
        host, _, ev = ent
        if lib().e4b_watch_device_error(ws.data_ptr(), host.data_ptr(), ev.cuda_event, stream_handle(ws.device)):
            self.raise_if_set(ws, what, host)

    def raise_if_set(self, ws: torch.Tensor, what: str, host: torch.Tensor | None = None) -> None:
        err = read_device_error(ws)  # synchronises: the copy queued before the clear has landed
        if host is not None:
            host.zero_()
        if err:
            raise E4BError(err, what + " (device error recorded by an earlier call on this workspace)")

    def check_all(self) -> None:
        for ws_ptr, (host, ws, ev) in list(self._w.items()):
            ev.synchronize()
            self.raise_if_set(ws, "check_errors", host)


error_watch = _ErrorWatch()


def check_errors() -> None:
    """Synchronise and raise ``E4BError`` if any watched workspace holds a device error."""
    error_watch.check_all()

