# SPDX-License-Identifier: Apache-2.0
"""Optional trace of QDQ calls: VLLM_QDQ_TRACE=1 prints the first 200.

Same output format as the reference (src/vllm_qdq_plugin/trace.py:9-16).
"""

from . import envs

TRACE_LIMIT = 200
_calls = 0


def trace_qdq(op_name: str, shape, dtype) -> None:
    if not envs.VLLM_QDQ_TRACE:
        return
    global _calls
    _calls += 1
    if _calls <= TRACE_LIMIT:
        print(f"[QDQ] op={op_name} shape={shape} dtype={dtype}")
