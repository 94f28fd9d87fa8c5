"""NF4-only stand-in for ``bitsandbytes.functional`` built on ``oracle.nf4``."""
import numpy as np
import torch

from oracle.nf4 import NF4_CODE, dequantize_nf4, quantize_nf4


class QuantState:
    def __init__(self, absmax=None, shape=None, code=None, blocksize=64, quant_type="nf4", dtype=None, **kw):
        self.absmax = absmax
        self.shape = shape
        self.code = code
        self.blocksize = blocksize
        self.quant_type = quant_type
        self.dtype = dtype


def get_4bit_type(typename, device=None, blocksize=64):
    if typename != "nf4":
        raise NotImplementedError("the oracle shim restates NF4 only")
    return torch.from_numpy(NF4_CODE.copy()).to(device if device is not None else "cpu")


def quantize_4bit(A, absmax=None, out=None, blocksize=64, compress_statistics=False, quant_type="nf4", quant_storage=torch.uint8):
    if quant_type != "nf4" or compress_statistics:
        raise NotImplementedError("the oracle shim restates NF4 without double-quant only")
    packed, am = quantize_nf4(A.detach().cpu(), blocksize)
    q = torch.from_numpy(packed).reshape(-1, 1).to(A.device)
    st = QuantState(absmax=torch.from_numpy(am).to(A.device), shape=A.shape,
                    code=get_4bit_type("nf4", A.device), blocksize=blocksize,
                    quant_type=quant_type, dtype=A.dtype)
    return q, st


def dequantize_4bit(A, quant_state=None, absmax=None, out=None, blocksize=64, quant_type="nf4"):
    qs = quant_state
    return dequantize_nf4(A.detach().cpu().numpy().reshape(-1), qs.absmax.detach().cpu().numpy().reshape(-1),
                          tuple(qs.shape), qs.dtype, qs.blocksize).to(A.device)


def create_dynamic_map(*a, **k):
    raise NotImplementedError("int8 codebook not restated")


def create_fp8_map(*a, **k):
    raise NotImplementedError("fp8 codebook not restated")
