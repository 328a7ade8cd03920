# SPDX-License-Identifier: Apache-2.0
"""MXFP8 activation quant-dequant (FP8 Marlin layers).

The reference applies MXFP8 QDQ (src/vllm_qdq_plugin/qdq/mxfp8.py:73-125) in
front of `float8_e4m3fn` Marlin GEMMs (src/vllm_qdq_plugin/patch.py:61-67,
:150-152).  That branch lies outside the FP4 hot path this package
accelerates, so this build raises instead of falling back to a CPU or
torch-op emulation.
"""

from __future__ import annotations

import torch


def mxfp8_qdq(x: torch.Tensor, group_size: int = 32) -> torch.Tensor:
    raise NotImplementedError(
        "vllm_qdq_plugin (B200): MXFP8 QDQ for float8_e4m3fn Marlin layers is not "
        "part of this build's FP4 hot path")
