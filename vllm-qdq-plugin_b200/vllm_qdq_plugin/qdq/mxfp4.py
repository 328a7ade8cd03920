# SPDX-License-Identifier: Apache-2.0
"""MXFP4 activation quant-dequant on B200 (sm_100a).

Drop-in for the reference's `vllm_qdq_plugin.qdq.mxfp4.mxfp4_qdq`
(reference: src/vllm_qdq_plugin/qdq/mxfp4.py:98-156): same signature, same
assertions, bit-identical output.  The work is one HBM pass in the C-ABI
kernel `qdq_mxfp4` (include/qdq_b200.h), registered as the torch.library op
`qdq_b200::mxfp4_qdq` so that dynamo/torch.compile graphs can trace the hook.
"""

from __future__ import annotations

import torch

from .. import _native


def _rows(x: torch.Tensor) -> torch.Tensor:
    # The kernel takes a row stride; only the element stride must be 1.
    return x if x.stride(-1) == 1 else x.contiguous()


@torch.library.custom_op("qdq_b200::mxfp4_qdq", mutates_args=())
def _mxfp4_qdq_op(x: torch.Tensor, group_size: int) -> torch.Tensor:
    _native.require_cuda(x)
    x = _rows(x)
    m, k = x.shape
    y = torch.empty((m, k), dtype=x.dtype, device=x.device)
    _native.call("qdq_mxfp4", x.data_ptr(), y.data_ptr(), None, None, m, k,
                 x.stride(0) if m > 1 else k, k, _native.DTYPE_CODE[x.dtype], group_size,
                 _native.stream_ptr(x.device))
    return y


@_mxfp4_qdq_op.register_fake
def _(x: torch.Tensor, group_size: int) -> torch.Tensor:
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("qdq_b200::mxfp4_quantize", mutates_args=())
def _mxfp4_quantize_op(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _native.require_cuda(x)
    x = _rows(x)
    m, k = x.shape
    kp = (k + 31) // 32 * 32
    codes = torch.empty((m, kp // 2), dtype=torch.uint8, device=x.device)
    scales = torch.empty((m, kp // 32), dtype=torch.uint8, device=x.device)
    _native.call("qdq_mxfp4", x.data_ptr(), None, codes.data_ptr(), scales.data_ptr(), m, k,
                 x.stride(0) if m > 1 else k, k, _native.DTYPE_CODE[x.dtype], 32,
                 _native.stream_ptr(x.device))
    return codes, scales


@_mxfp4_quantize_op.register_fake
def _(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    kp = (k + 31) // 32 * 32
    return (x.new_empty((m, kp // 2), dtype=torch.uint8),
            x.new_empty((m, kp // 32), dtype=torch.uint8))


def mxfp4_qdq(x: torch.Tensor, group_size: int = 32) -> torch.Tensor:
    """Quantize-dequantize input to MXFP4 (E2M1 + E8M0 scales).

    Args:
        x: 2D tensor [M, K] in bf16/fp16 (CUDA)
        group_size: number of elements per scale group (32)

    Returns:
        Tensor same shape and dtype as x, with MXFP4 quantization noise applied.
    """
    orig_dtype = x.dtype
    assert x.dim() == 2, (
        f"mxfp4_qdq only supports 2D tensors for now, but got {x.dim()}D"
    )
    assert orig_dtype in (torch.float16, torch.bfloat16), (
        f"mxfp4_qdq only supports fp16/bf16 tensors, but got {orig_dtype}"
    )
    return torch.ops.qdq_b200.mxfp4_qdq(x, group_size)


def mxfp4_quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """MXFP4 codes of the same quantisation `mxfp4_qdq` applies.

    Returns (codes [M, Kp/2] uint8, element 2j in the low nibble of byte j;
    scales [M, Kp/32] uint8 E8M0), Kp = K rounded up to 32.  Dequantising
    them reproduces `mxfp4_qdq(x)` exactly.
    """
    assert x.dim() == 2 and x.dtype in (torch.float16, torch.bfloat16)
    return torch.ops.qdq_b200.mxfp4_quantize(x)
