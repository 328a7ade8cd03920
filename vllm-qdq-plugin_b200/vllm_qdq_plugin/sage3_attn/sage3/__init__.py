# SPDX-License-Identifier: Apache-2.0
"""sage3 — SageAttention3-style FP4 attention on B200 tensor cores.

Public API (same names as the reference package
src/vllm_qdq_plugin/sage3_attn/sage3/__init__.py):
    sageattn3_standalone()               config-based entry point (HND tensors)
    sageattn3_torch_triton_standalone()  backward-compatible entry point
    scaled_dot_product_attention()       SDPA-compatible wrapper
    ATTENTION_CONFIGS, ACC_DTYPE_MAP     config names / accumulator modes
"""

from .api import (
    ACC_DTYPE_MAP,
    ATTENTION_CONFIGS,
    sage3_attention_nhd,
    sageattn3_standalone,
    sageattn3_torch_triton_standalone,
    scaled_dot_product_attention,
)

__all__ = [
    "sageattn3_standalone",
    "sageattn3_torch_triton_standalone",
    "scaled_dot_product_attention",
    "sage3_attention_nhd",
    "ATTENTION_CONFIGS",
    "ACC_DTYPE_MAP",
]
