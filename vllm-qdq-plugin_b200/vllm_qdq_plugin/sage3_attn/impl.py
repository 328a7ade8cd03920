# SPDX-License-Identifier: Apache-2.0
"""Sage3 attention implementation for vllm-omni diffusion models (sm_100a).

Same surface as the reference (src/vllm_qdq_plugin/sage3_attn/impl.py:26-137):
  __init__(num_heads, head_size, softmax_scale, causal=False, num_kv_heads=None,
           prefix="", backend_kwargs=None, **extra)
  forward_cuda(query, key, value, attn_metadata=None, *, config_override=None)
  _forward_sdpa(query, key, value)       (cross-attention / routed fallback)
  _forward_sage3(query, key, value, config=None)
Inputs and output are NHD [B, N, H, D].  The reference transposes Q/K/V to
HND with three copies; here the kernels read the NHD strides directly and
write the NHD output.
"""

from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from .. import envs
from .._log import init_logger
from .sage3.api import sage3_attention_nhd, unsupported_reason

logger = init_logger(__name__)
_WARNED: set[str] = set()


def _warn_once(msg: str) -> None:
    if msg not in _WARNED:
        _WARNED.add(msg)
        logger.warning("Sage3 FP4 attention: %s; this call runs SDPA instead", msg)

try:
    from vllm_omni.diffusion.attention.backends.abstract import AttentionImpl, AttentionMetadata
except ImportError:  # standalone use / tests
    class AttentionImpl:  # type: ignore[no-redef]
        pass

    AttentionMetadata = object  # type: ignore[misc,assignment]


class Sage3TritonImpl(AttentionImpl):
    """SAGE_ATTN implementation using the sm_100a FP4 attention kernels."""

    def __init__(self, num_heads: int, head_size: int, softmax_scale: float, causal: bool = False,
                 num_kv_heads: int | None = None, prefix: str = "", backend_kwargs: dict | None = None,
                 **extra_impl_args) -> None:
        self.causal = causal
        self.softmax_scale = softmax_scale
        self._config = envs.SAGE3_QUANT_FORMAT
        self._acc_dtype = envs.SAGE3_ACC_DTYPE
        if backend_kwargs:
            self._config = backend_kwargs.pop("sage3_config", self._config)
            self._acc_dtype = backend_kwargs.pop("sage3_acc_dtype", self._acc_dtype)
            if backend_kwargs:
                logger.warning("Sage3TritonImpl ignoring backend_kwargs: %s", list(backend_kwargs.keys()))

    def forward_cuda(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     attn_metadata: AttentionMetadata = None, *,
                     config_override: str | None = None) -> torch.Tensor:
        # Cross-attention (different Q and K/V lengths) goes to SDPA, as in the reference.
        if query.shape[1] != key.shape[1]:
            return self._forward_sdpa(query, key, value)
        # The backend advertises the reference's head sizes (32-256); the FP4
        # kernels take the head dims and dtypes in sage3.api.SUPPORTED_*.  A call
        # outside them runs SDPA, with one warning per (head dim, dtype).
        why = unsupported_reason(query)
        if why is not None:
            _warn_once(why)
            return self._forward_sdpa(query, key, value)
        return self._forward_sage3(query, key, value, config=config_override or self._config)

    def _forward_sdpa(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
        """SDPA fallback for cross-attention (N_q != N_k); NHD in and out."""
        out = F.scaled_dot_product_attention(query.transpose(1, 2), key.transpose(1, 2),
                                             value.transpose(1, 2), scale=self.softmax_scale,
                                             is_causal=False)
        return out.transpose(1, 2)

    @torch.compiler.disable()
    def _forward_sage3(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                       config: str | None = None) -> torch.Tensor:
        cfg = config or self._config
        if os.environ.get("SAGE3_DUMP_INPUTS", "0") == "1":
            self._dump(query, key, value, cfg)
        return sage3_attention_nhd(query, key, value, config=cfg, is_causal=self.causal,
                                   sm_scale=self.softmax_scale, acc_dtype=self._acc_dtype)

    def _dump(self, query, key, value, cfg) -> None:
        """SAGE3_DUMP_INPUTS / SAGE3_DUMP_DIR / SAGE3_DUMP_MAX: save HND inputs
        for offline analysis (reference impl.py:106-126)."""
        dump_dir = os.environ.get("SAGE3_DUMP_DIR", "/tmp/sage3_inputs")
        os.makedirs(dump_dir, exist_ok=True)
        count = getattr(self, "_dump_count", 0)
        if count >= int(os.environ.get("SAGE3_DUMP_MAX", "1")):
            return
        q, k, v = (t.transpose(1, 2) for t in (query, key, value))
        path = os.path.join(dump_dir, f"self_attn_input_{count}.pt")
        torch.save({"q": q.cpu(), "k": k.cpu(), "v": v.cpu(), "sm_scale": self.softmax_scale,
                    "is_causal": self.causal, "config": cfg, "acc_dtype": self._acc_dtype,
                    "q_shape": list(q.shape)}, path)
        logger.info("Dumped self-attention inputs to %s", path)
        self._dump_count = count + 1
