# SPDX-License-Identifier: Apache-2.0
"""Sage3 FP4 attention for the vllm-omni SAGE_ATTN backend slot (sm_100a)."""
