# SPDX-License-Identifier: Apache-2.0
"""Per-(layer, step) routing hook on vllm-omni's attention module.

Wraps `vllm_omni.diffusion.attention.layer.Attention._run_local_attention`
(reference: src/vllm_qdq_plugin/sage3_attn/routing/patch_attention.py): the
layer index lives on the module and the denoising step on vllm-omni's forward
context, so the wrapper resolves the route there and calls the Sage3 impl with
`config_override` (or its SDPA path for "sdpa").  Anything it does not route
(fp32 inputs, cross-attention, another backend, no matching rule) goes to the
original method unchanged.
"""

from __future__ import annotations

import torch

from ..._log import init_logger
from ..impl import Sage3TritonImpl
from .route_table import SDPA_TOKEN, RouteTable

logger = init_logger(__name__)

try:  # vllm-omni's forward context (absent outside a diffusion worker)
    from vllm_omni.diffusion.forward_context import get_forward_context, is_forward_context_available
except ImportError:  # pragma: no cover - depends on the environment
    def is_forward_context_available() -> bool:
        return False

    def get_forward_context():
        raise RuntimeError("vllm-omni forward context unavailable")

_installed = False
_ORIG = None
_TABLE: RouteTable | None = None
_DEBUG = False
_seen: set = set()


def _debug_log(layer_idx, step, route) -> None:
    key = (layer_idx, step, route)
    if key not in _seen:
        _seen.add(key)
        logger.warning("sage3 route: layer=%s step=%s -> %s", layer_idx, step, route)


def _routed_run_local_attention(self, query, key, value, attn_metadata):
    return _dispatch(self, query, key, value, attn_metadata)


@torch.compiler.disable()
def _dispatch(self, query, key, value, attn_metadata):
    if query.dtype == torch.float32:                      # the original's fp32 -> SDPA path
        return _ORIG(self, query, key, value, attn_metadata)
    impl = self.attention
    if self.role != "self" or not isinstance(impl, Sage3TritonImpl):
        return _ORIG(self, query, key, value, attn_metadata)
    step = get_forward_context().denoise_step_idx if is_forward_context_available() else None
    route = _TABLE.resolve(self.layer_idx, step)
    if route is None:
        return _ORIG(self, query, key, value, attn_metadata)
    if _DEBUG:
        _debug_log(self.layer_idx, step, route)
    if route == SDPA_TOKEN:
        return impl._forward_sdpa(query, key, value)
    return impl.forward_cuda(query, key, value, attn_metadata, config_override=route)


def install(route_file: str) -> None:
    """Load the route file and wrap the attention module's dispatch; idempotent.
    A bad route file raises ValueError and leaves the module untouched."""
    global _installed, _ORIG, _TABLE, _DEBUG
    if _installed:
        return
    from ... import envs
    table = RouteTable.from_json_file(route_file)      # validate before patching anything
    from vllm_omni.diffusion.attention.layer import Attention
    _TABLE = table
    _DEBUG = bool(envs.SAGE3_ROUTE_DEBUG)
    _ORIG = Attention._run_local_attention
    Attention._run_local_attention = _routed_run_local_attention
    _installed = True
    logger.warning("sage3 per-(layer, step) attention routing installed from %s (default=%s, %d rule(s))",
                   route_file, table.default, len(table))
