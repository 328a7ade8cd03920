# SPDX-License-Identifier: Apache-2.0
"""SAGE_ATTN diffusion-attention backend (vllm-omni) backed by the sm_100a
FP4 attention.  Same class name, name and head sizes as the reference
(src/vllm_qdq_plugin/sage3_attn/backend.py:9-30), so registration through
`register_omni()` is a drop-in.
"""

from __future__ import annotations

try:  # vllm-omni provides the base class in a serving process
    from vllm_omni.diffusion.attention.backends.abstract import AttentionBackend
except ImportError:  # standalone use / tests: a minimal stand-in with the same surface
    class AttentionBackend:  # type: ignore[no-redef]
        accept_output_buffer: bool = False


class Sage3TritonBackend(AttentionBackend):
    """Out-of-tree sage3 attention backend (the name is the reference's; the
    kernels are hand-written sm_100a CUDA, not Triton)."""

    accept_output_buffer: bool = False

    @staticmethod
    def get_supported_head_sizes() -> list[int]:
        return [32, 64, 96, 128, 160, 192, 224, 256]

    @staticmethod
    def get_name() -> str:
        return "SAGE_ATTN"

    @staticmethod
    def get_impl_cls() -> type:
        from .impl import Sage3TritonImpl

        return Sage3TritonImpl
