# SPDX-License-Identifier: Apache-2.0
"""vllm-qdq-plugin, B200-native build.

Entry points (same names as the reference, src/vllm_qdq_plugin/__init__.py and
pyproject.toml:8-12):
  vllm.general_plugins:      qdq        = vllm_qdq_plugin:register
  vllm_omni.general_plugins: sage3_attn = vllm_qdq_plugin:register_omni

`register()` (every vLLM process) installs the activation-QDQ wrappers on the
Marlin ops when VLLM_QDQ=1.  `register_omni()` (diffusion workers) overrides
the SAGE_ATTN backend slot with the sm_100a FP4 attention when
VLLM_SAGE3_TRITON=1.  Underneath, every hook calls hand-written sm_100a CUDA
through the C ABI of libqdq_b200.so (include/qdq_b200.h).
"""

from __future__ import annotations

from . import envs
from ._log import init_logger

logger = init_logger(__name__)

SAGE3_BACKEND_PATH = "vllm_qdq_plugin.sage3_attn.backend.Sage3TritonBackend"


def register():
    """vLLM plugin hook, run in the main process and in every worker."""
    if not envs.VLLM_QDQ:
        return
    from .patch import apply_patches

    apply_patches()
    logger.info("vllm-qdq-plugin: patches applied (VLLM_QDQ enabled)")


def _register_sage_attn_slot(backend_path: str, what: str, flag: str) -> bool:
    try:
        from vllm_omni.diffusion.attention.backends.registry import (
            DiffusionAttentionBackendEnum,
            register_diffusion_backend,
        )
    except ImportError as e:
        logger.warning("vllm-qdq-plugin: cannot register %s backend — vllm_omni not "
                       "available (%s)", what, e)
        return False
    register_diffusion_backend(DiffusionAttentionBackendEnum.SAGE_ATTN, backend_path)
    logger.warning("vllm-qdq-plugin: registered %s backend as SAGE_ATTN (%s=1)", what, flag)
    return True


def register_omni_sage3_triton():
    return _register_sage_attn_slot(SAGE3_BACKEND_PATH, "sage3 (sm_100a FP4)", "VLLM_SAGE3_TRITON")


def _maybe_install_route(route_file: str) -> None:
    """Per-(layer, step) attention routing from SAGE3_ROUTE_FILE (reference
    __init__.py:110-127); a bad route file or a missing vllm-omni logs and
    leaves routing off instead of stopping the worker."""
    if not route_file:
        return
    try:
        from .sage3_attn.routing import patch_attention
        patch_attention.install(route_file)
    except Exception as e:  # noqa: BLE001 - startup must continue
        logger.warning("vllm-qdq-plugin: failed to install sage3 attention routing from %s (%s) — "
                       "continuing without routing", route_file, e)


def _not_in_this_build(what: str, flag: str) -> None:
    # SpargeAttn and the external SageAttention3 CuTe kernel are outside the
    # attention this build replaces.
    logger.warning("vllm-qdq-plugin (B200 build): %s=1 requests %s, which this build does "
                   "not provide; the SAGE_ATTN slot is left unchanged", flag, what)


def register_omni():
    """vllm-omni plugin hook (diffusion workers).

    SpargeAttn and sage3 share the SAGE_ATTN slot; SpargeAttn wins when both
    are requested (reference __init__.py:137-165).
    """
    sage3_requested = envs.VLLM_SAGE3_TRITON or envs.VLLM_SAGE3_CUTE
    if envs.VLLM_SPARGE_ATTN and sage3_requested:
        logger.warning("vllm-qdq-plugin: both VLLM_SPARGE_ATTN and a sage3 flag are set; "
                       "they share the SAGE_ATTN backend slot. Using SpargeAttn.")
    if envs.VLLM_SPARGE_ATTN:
        _not_in_this_build("the SpargeAttn backend", "VLLM_SPARGE_ATTN")
    elif envs.VLLM_SAGE3_TRITON:
        register_omni_sage3_triton()
        _maybe_install_route(envs.SAGE3_ROUTE_FILE)
    elif envs.VLLM_SAGE3_CUTE:
        _not_in_this_build("the external SageAttention3 CuTe kernel", "VLLM_SAGE3_CUTE")
    else:
        logger.warning("vllm-qdq-plugin: no sage3 backend registered for vllm-omni — set "
                       "VLLM_SAGE3_TRITON=1 or VLLM_SAGE3_CUTE=1 to enable")
