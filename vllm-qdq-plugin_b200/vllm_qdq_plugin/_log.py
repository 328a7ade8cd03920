# SPDX-License-Identifier: Apache-2.0
"""Logger factory: vLLM's `init_logger` when vLLM is importable, else stdlib
logging with a `warning_once` helper (the reference always runs inside vLLM,
src/vllm_qdq_plugin/__init__.py:8-12)."""

from __future__ import annotations

import logging


def init_logger(name: str):
    try:
        from vllm.logger import init_logger as vllm_init_logger
        return vllm_init_logger(name)
    except Exception:
        logger = logging.getLogger(name)
        seen: set[str] = set()

        def warning_once(msg, *args):
            key = msg % args if args else msg
            if key not in seen:
                seen.add(key)
                logger.warning(msg, *args)

        logger.warning_once = warning_once  # type: ignore[attr-defined]
        return logger
