"""CPU: the C oracle is pinned to the reference's own outputs.

The fixtures in tests/golden/ were produced by running the reference
(tests/golden/make_golden.py): the plugin's mxfp4_qdq and mxfp8_qdq, vLLM
0.22's ref_nvfp4_quant_dequant (CPU branch) and the plugin's
quantize_to_mxfp4.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import qdq as oq


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("subset", ["natural", "context", "c1_slice", "odd_k"])
def test_mxfp4_oracle_matches_reference(tag, subset):
    d = golden(f"mxfp4_{tag}.npz")
    y = oq.mxfp4_qdq(d[f"{subset}_x"], fp16=(tag == "fp16"))
    np.testing.assert_array_equal(y, d[f"{subset}_y"])


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("subset", ["natural", "context", "c1_slice", "odd_k"])
def test_mxfp8_oracle_matches_reference(tag, subset):
    d = golden(f"mxfp8_{tag}.npz")
    y = oq.mxfp8_qdq(d[f"{subset}_x"], fp16=(tag == "fp16"))
    np.testing.assert_array_equal(y, d[f"{subset}_y"])


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
def test_nvfp4_oracle_matches_reference(tag):
    d = golden(f"nvfp4_{tag}.npz")
    checked = 0
    for key in d.files:
        if not key.endswith("_y"):
            continue
        base = key[:-2]
        gs = d["c2_slice_gs"][0] if base == "c2_slice" else d["gs" + base.split("_gs")[1]][0]
        y = oq.nvfp4_qdq(d[base + "_x"], float(gs), fp16=(tag == "fp16"))
        np.testing.assert_array_equal(y, d[key], err_msg=base)
        checked += 1
    assert checked >= 10


def test_mxfp4_hw_quant_oracle_matches_reference():
    d = golden("mxfp4_hw_quant.npz")
    for name in ("qk", "v"):
        codes, scales = oq.mxfp4_hw_quant(d[f"{name}_x"])
        np.testing.assert_array_equal(codes, d[f"{name}_codes"])
        np.testing.assert_array_equal(scales, d[f"{name}_scales"])


def test_mxfp8_hw_quant_oracle_matches_reference():
    """quantize_to_mxfp8 (sage3/mxfp8_hw_kernel.py:37): E4M3 codes (including
    -0 codes) and E8M0 bytes (including the 1e-12 clamp and exact powers of
    two) equal the reference's."""
    d = golden("mxfp8_hw_quant.npz")
    for name in ("qk", "v"):
        codes, scales = oq.mxfp8_hw_quant(d[f"{name}_x"])
        np.testing.assert_array_equal(codes, d[f"{name}_codes"])
        np.testing.assert_array_equal(scales, d[f"{name}_scales"])


def test_e4m3_rounding_matches_torch_cast():
    # the NVFP4 block scale is torch's fp32 -> float8_e4m3fn -> fp32 cast
    g = torch.Generator().manual_seed(0)
    vals = torch.cat([
        torch.rand(20000, generator=g) * 448.0,
        torch.exp2(torch.rand(20000, generator=g) * 20 - 14),
        torch.arange(0, 2 ** -6, 2 ** -12),               # subnormal grid and midpoints
        torch.tensor([0.0, 448.0, 2 ** -9, 1.5 * 2 ** -10, 2 ** -10, 0.9 * 2 ** -10, 240.0,
                      232.0, 248.0, 1.0625, 1.1875]),
    ]).float()
    ref = vals.to(torch.float8_e4m3fn).to(torch.float32).numpy()
    ours = np.array([oq.round_e4m3(float(v)) for v in vals.numpy()], np.float32)
    np.testing.assert_array_equal(ours, ref)


def test_codes_dequantise_to_qdq_output():
    d = golden("mxfp4_bf16.npz")
    x = d["c1_slice_x"]
    y, codes, scales = oq.mxfp4_qdq(x, codes=True)
    lut = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float32)
    vals = np.stack([lut[codes & 15], lut[codes >> 4]], -1).reshape(x.shape)
    deq = vals * np.exp2(np.repeat(scales.astype(np.float32) - 127, 32, axis=1))
    ybits = (y.astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(deq, ybits)
