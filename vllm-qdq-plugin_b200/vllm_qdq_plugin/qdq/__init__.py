# SPDX-License-Identifier: Apache-2.0
"""QDQ (quant-dequant) hooks: `(x, **config) -> Tensor`, same shape and dtype.

Mirrors the reference's `vllm_qdq_plugin.qdq` package
(reference: src/vllm_qdq_plugin/qdq/__init__.py).
"""

from .host import qdq_from_host
from .mxfp4 import mxfp4_qdq, mxfp4_quantize
from .mxfp8 import mxfp8_qdq, mxfp8_quantize
from .nvfp4 import nvfp4_global_scale, nvfp4_qdq, nvfp4_quantize

__all__ = ["mxfp4_qdq", "mxfp8_qdq", "nvfp4_qdq", "mxfp4_quantize", "mxfp8_quantize", "nvfp4_quantize",
           "nvfp4_global_scale", "qdq_from_host"]
