"""CPU: the attention oracle (oracle/attn.py) against the reference's own outputs.

tests/golden/attn_reference.npz holds outputs of the unmodified reference run
under Triton's interpreter (tests/golden/make_attn_golden.py).  For the
hardware configs the oracle restates the reference's kernel step for step
(sage3/mxfp4_hw_kernel.py:167-393, sage3/mxfp8_hw_kernel.py:100-246), so run at
the reference's 64-key tile with its padding keys attended it must agree to
the bf16 rounding of the reference's output (relative L2 2^-9.2 ~ 0.0017;
fp16 inputs give an fp16 output, rounded more finely).
For the emulated configs the oracle states this build's definition (real
E2M1 codes where the reference fake-quantises on a 9-level grid), so only its
accuracy is held against the reference's: err <= 1.1 * err(reference) + 0.005
against float64 attention.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import attn as oa

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_attn_golden as G  # noqa: E402  (inputs and case table; no reference import)


def _case(name):
    fx = golden("attn_reference.npz")
    q, k, v = G.case_inputs(name)
    assert G.input_checksum(q, k, v) == str(fx[f"{name}/checksum"])
    rows = fx[f"{name}/rows"]
    ref = oa.bits_to_f32(fx[f"{name}/out"], q.dtype == torch.float16).astype(np.float64)
    return q, k, v, rows, ref


@pytest.mark.parametrize("name", ["mxfp4_hw_L1024", "mxfp8_hw_L1024", "mxfp4_hw_D64_L1024", "mxfp4_hw_L75600",
                                  "mxfp4_hw_f16_L1024", "mxfp8_hw_f16_L1024"])
def test_hardware_config_oracle_reproduces_reference(name):
    config = G.CASES[name][0]
    q, k, v, rows, ref = _case(name)
    f16 = q.dtype == torch.float16
    if len(rows) < q.shape[2]:
        # the full config-4 sequence: the last, ragged query tile (80 rows) is
        # checked here (its keys include the reference's 48 zero padding keys);
        # the GPU test covers all three tiles of the fixture
        last = rows >= rows.max() // 128 * 128
        rows, ref = rows[last], ref[:, :, last]
    for h in range(q.shape[1]):
        bits = [t[0, h].contiguous().view(torch.int16).numpy().view(np.uint16)[:, None, :] for t in (q, k, v)]
        if len(rows) < q.shape[2]:
            got = oa.attention_rows(*bits, 1.0 / math.sqrt(q.shape[-1]), rows, config=config,
                                    block_n=oa.REF_BLOCK_N[config], mask_padding=False, f16=f16)
        else:
            got = oa.attention(*bits, 1.0 / math.sqrt(q.shape[-1]), config=config, block_n=oa.REF_BLOCK_N[config],
                               mask_padding=False, f16=f16)[:, 0]
        assert oa.rel_l2(got, ref[0, h]) < 2.2e-3, (name, h, oa.rel_l2(got, ref[0, h]))


@pytest.mark.parametrize("name", ["mxfp4_L1024", "nvfp4_bf16pv_L1024", "nvfp4_D64_L1024", "nvfp4_f16pv_L1024"])
def test_emulated_config_oracle_accuracy_against_reference(name):
    config = G.CASES[name][0]
    q, k, v, rows, ref = _case(name)
    f16 = q.dtype == torch.float16
    for h in range(q.shape[1]):
        bits = [t[0, h].contiguous().view(torch.int16).numpy().view(np.uint16)[:, None, :] for t in (q, k, v)]
        ex = oa.exact_attention(*bits, 1.0 / math.sqrt(q.shape[-1]), f16=f16)[:, 0]
        got = oa.attention(*bits, 1.0 / math.sqrt(q.shape[-1]), config=config, block_n=128, f16=f16)[:, 0]
        e_ref, e_got = oa.rel_l2(ref[0, h], ex), oa.rel_l2(got, ex)
        assert e_got <= 1.1 * e_ref + 0.005, (name, h, e_got, e_ref)
