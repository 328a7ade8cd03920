# SPDX-License-Identifier: Apache-2.0
"""Environment knobs of the plugin, evaluated lazily on every attribute access.

Same names, defaults and validation as the reference's lazy env module
(reference: src/vllm_qdq_plugin/envs.py:21-131): truthy flags accept
"1"/"true"/"yes" (any case); choice-valued knobs are validated against their
allowed values, optionally case-insensitively, and return the canonical
spelling.
"""

from __future__ import annotations

import os
from collections.abc import Callable
from typing import Any

_TRUTHY = ("1", "true", "yes")


def _flag(name: str, default: str = "0") -> Callable[[], bool]:
    return lambda: os.getenv(name, default).lower() in _TRUTHY


def _str(name: str, default: str) -> Callable[[], str]:
    return lambda: os.getenv(name, default)


def env_with_choices(
    env_name: str,
    default: str | None,
    choices: list[str] | Callable[[], list[str]],
    case_sensitive: bool = True,
) -> Callable[[], str | None]:
    """Return a getter that validates `env_name` against `choices`.

    Unset -> `default`.  A value outside `choices` raises ValueError naming the
    variable and the valid options.  With case_sensitive=False the canonical
    spelling from `choices` is returned.
    """

    def getter() -> str | None:
        raw = os.getenv(env_name)
        if raw is None:
            return default
        allowed = list(choices() if callable(choices) else choices)
        if case_sensitive:
            if raw in allowed:
                return raw
        else:
            for choice in allowed:
                if choice.lower() == raw.lower():
                    return choice
        raise ValueError(
            f"Invalid value '{raw}' for {env_name}. Valid options: {allowed}.")

    return getter


# SAGE3_QUANT_FORMAT / SAGE3_ACC_DTYPE keep the reference's free-form strings
# (validated where they are used, as the reference does).
environment_variables: dict[str, Callable[[], Any]] = {
    "VLLM_QDQ_TRACE": _flag("VLLM_QDQ_TRACE"),
    "VLLM_QDQ": _flag("VLLM_QDQ"),
    "VLLM_MARLIN_MOE_QDQ_MODE": env_with_choices(
        "VLLM_MARLIN_MOE_QDQ_MODE", default="0", choices=["0", "FORCE_MXFP4"],
        case_sensitive=False),
    "VLLM_SAGE3_TRITON": _flag("VLLM_SAGE3_TRITON"),
    "VLLM_SAGE3_CUTE": _flag("VLLM_SAGE3_CUTE"),
    "SAGE3_QUANT_FORMAT": _str("SAGE3_QUANT_FORMAT", "mxfp4"),
    "SAGE3_ACC_DTYPE": _str("SAGE3_ACC_DTYPE", "fp32"),
    "SAGE3_ROUTE_FILE": _str("SAGE3_ROUTE_FILE", ""),
    "SAGE3_ROUTE_DEBUG": _flag("SAGE3_ROUTE_DEBUG"),
    "VLLM_SPARGE_ATTN": _flag("VLLM_SPARGE_ATTN"),
    "SPARGE_ATTN_REPO": _str("SPARGE_ATTN_REPO", ""),
    "SPARGE_MODE": env_with_choices(
        "SPARGE_MODE", default="topk", choices=["topk", "cdfthreshd"], case_sensitive=False),
    "SPARGE_TOPK": _str("SPARGE_TOPK", "1.0"),
    "SPARGE_CDFTHRESHD": _str("SPARGE_CDFTHRESHD", "0.98"),
    # B200 build: use the fused FP4 tcgen05 GEMM for Marlin layers whose raw
    # MXFP4 weights were captured (see vllm_qdq_plugin.gemm); "0" keeps the
    # reference behaviour (QDQ then the original Marlin kernel).
    "VLLM_QDQ_FUSED_GEMM": _flag("VLLM_QDQ_FUSED_GEMM"),
    # B200 build: on NVFP4 Marlin layers (float4_e2m1f weights with a global
    # scale, which vLLM passes only for NVFP4: marlin_utils_fp4.py
    # apply_fp4_marlin_linear), quantise the activation as NVFP4 (group 16,
    # E4M3 block scales, per-tensor gs = 448*6/amax) instead of the reference's
    # MXFP4 QDQ.  "0" keeps the reference behaviour.
    "VLLM_QDQ_NVFP4_ACT": _flag("VLLM_QDQ_NVFP4_ACT"),
}


def __getattr__(name: str):
    if name in environment_variables:
        return environment_variables[name]()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return list(environment_variables.keys())


def is_set(name: str) -> bool:
    """True when the variable is explicitly present in the environment."""
    if name in environment_variables:
        return name in os.environ
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
