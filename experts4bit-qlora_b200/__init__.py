"""experts4bit-b200: the fused-expert forward of experts4bit-qlora, B200-native.

Drop-in names (same constructors, state_dict layout and patch semantics as the
reference's ``experts4bit_qlora`` package): ``ExpertsNbit``, ``Experts4bit``,
``ExpertsLoRA``, ``enable_fast``, ``disable_fast``, ``fast_available``,
``enable_fast_train``, ``disable_fast_train``, ``normalize_quant_type``. The hot path is libe4b.so (hand-written sm_100a CUDA
behind the C ABI in include/e4b.h), reached through ctypes.

The package directory is named ``experts4bit-qlora_b200``; import it with
``importlib.import_module("experts4bit-qlora_b200")``. After that first import
it is also registered as ``experts4bit_qlora_b200``.
"""
import sys as _sys

from . import _native, ep, mxfp4, ops  # noqa: F401
from ._native import check_errors
from .experts import Experts4bit, ExpertsNbit, normalize_quant_type
from .fast import disable_fast, enable_fast, fast_available
from .fp8_experts import ExpertsFp8Blocks
from .mxfp4 import ExpertsMxfp4
from .ep import ExpertParallelMoE, PeerExchange, shard_experts
from .lora import ExpertsLoRA
from .train import disable_fast_train, enable_fast_train
from .router import route, TopKRouter
from .residency import (disable_hot_residency, disable_pipelined_residency, dispatched_modules,
                        enable_hot_residency, enable_pipelined_residency, target_modules)

__version__ = "0.1.0"

__all__ = [
    "Experts4bit", "ExpertsNbit", "ExpertsLoRA", "enable_fast", "disable_fast", "fast_available",
    "normalize_quant_type", "check_errors", "enable_fast_train", "disable_fast_train", "route", "TopKRouter", "ops", "ExpertParallelMoE", "PeerExchange", "shard_experts", "ExpertsFp8Blocks",
    "ExpertsMxfp4", "enable_hot_residency", "disable_hot_residency", "enable_pipelined_residency", "disable_pipelined_residency",
    "target_modules", "dispatched_modules",
]

_sys.modules.setdefault("experts4bit_qlora_b200", _sys.modules[__name__])
