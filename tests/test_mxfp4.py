"""MXFP4 dequantization: the oracle restatement and the library against the reference's
own ``dequantize_mxfp4`` outputs (tests/golden/mxfp4.npz, made by
tests/golden/make_mxfp4_golden.py), bit for bit in bf16, fp16 and fp32."""
import importlib
import os

import numpy as np
import pytest
import torch

from oracle import mxfp4 as OM

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "mxfp4.npz"))
DTYPES = [(torch.bfloat16, "bf16", torch.int16), (torch.float16, "f16", torch.int16), (torch.float32, "f32", torch.int32)]


def _bits(t, view):
    return t.contiguous().view(view).cpu().numpy()


@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_oracle_matches_reference(case, dt, tag, view):
    v = OM.dequantize_mxfp4_f32(G[f"{case}_blocks"], G[f"{case}_scales"])
    got = torch.from_numpy(v).to(dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_host_library_matches_reference(e4b, case, dt, tag, view):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    got = mx.dequantize_mxfp4(torch.from_numpy(G[f"{case}_blocks"]), torch.from_numpy(G[f"{case}_scales"]), dtype=dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


def test_byte_reinterpretation_and_shape_errors(e4b):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    b, s = torch.from_numpy(G["single_blocks"]), torch.from_numpy(G["single_scales"])
    ref = mx.dequantize_mxfp4(b, s)
    assert torch.equal(mx.dequantize_mxfp4(b.view(torch.int8), s), ref)  # int8-labelled blocks: same bytes
    with pytest.raises(ValueError):
        mx.dequantize_mxfp4(b, s[:, :1])
    with pytest.raises(ValueError):
        mx.dequantize_mxfp4(b[0], s[0])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_device_kernel_matches_reference(e4b, case, dt, tag, view):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    got = mx.dequantize_mxfp4(torch.from_numpy(G[f"{case}_blocks"]).cuda(),
                              torch.from_numpy(G[f"{case}_scales"]).cuda(), dtype=dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


def test_scales_on_another_device_are_refused(e4b):
    """Scales on another device than the blocks are refused before any pointer reaches a kernel."""
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    b, s = torch.from_numpy(G["single_blocks"]), torch.from_numpy(G["single_scales"])
    with pytest.raises(ValueError, match="blocks on"):
        mx.dequantize_mxfp4(b, s.to("meta"))


def test_scale_255_follows_ldexp():
    """e8m0 255 is 2**128: 0.5 * 2**128 stays finite, codes >= 1 overflow, zero codes stay zeros."""
    blocks = np.array([[[0x10, 0x8A]]], dtype=np.uint8)   # codes (lo, hi): 0, 0.5 | -1.0, -0.0
    v = OM.dequantize_mxfp4_f32(blocks, np.array([[255]], dtype=np.uint8)).reshape(-1)
    assert v[0] == 0 and not np.signbit(v[0])
    assert v[1] == np.float32(2.0 ** 127)
    assert v[2] == -np.inf
    assert v[3] == 0 and np.signbit(v[3])
