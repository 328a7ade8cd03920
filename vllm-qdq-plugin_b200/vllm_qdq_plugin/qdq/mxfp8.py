# SPDX-License-Identifier: Apache-2.0
"""MXFP8 activation quant-dequant on B200 (sm_100a), for float8_e4m3fn Marlin layers.

Drop-in for the reference's `vllm_qdq_plugin.qdq.mxfp8.mxfp8_qdq`
(reference: src/vllm_qdq_plugin/qdq/mxfp8.py:73-125, applied at
src/vllm_qdq_plugin/patch.py:61-67 and :150-152): same signature, same
assertions, bit-identical output.  The work is one HBM pass in the C-ABI
kernel `qdq_mxfp8` (include/qdq_b200.h), registered as the torch.library op
`qdq_b200::mxfp8_qdq`.
"""

from __future__ import annotations

import torch

from .. import _native


def _rows(x: torch.Tensor) -> torch.Tensor:
    # The kernel takes a row stride; only the element stride must be 1.
    return x if x.stride(-1) == 1 else x.contiguous()


@torch.library.custom_op("qdq_b200::mxfp8_qdq", mutates_args=())
def _mxfp8_qdq_op(x: torch.Tensor, group_size: int) -> torch.Tensor:
    _native.require_cuda(x)
    x = _rows(x)
    m, k = x.shape
    y = torch.empty((m, k), dtype=x.dtype, device=x.device)
    _native.call("qdq_mxfp8", x.data_ptr(), y.data_ptr(), None, None, m, k,
                 x.stride(0) if m > 1 else k, k, _native.DTYPE_CODE[x.dtype], group_size,
                 _native.stream_ptr(x.device))
    return y


@_mxfp8_qdq_op.register_fake
def _(x: torch.Tensor, group_size: int) -> torch.Tensor:
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("qdq_b200::mxfp8_quantize", mutates_args=())
def _mxfp8_quantize_op(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _native.require_cuda(x)
    x = _rows(x)
    m, k = x.shape
    kp = (k + 31) // 32 * 32
    codes = torch.empty((m, kp), dtype=torch.uint8, device=x.device)
    scales = torch.empty((m, kp // 32), dtype=torch.uint8, device=x.device)
    _native.call("qdq_mxfp8", x.data_ptr(), None, codes.data_ptr(), scales.data_ptr(), m, k,
                 x.stride(0) if m > 1 else k, k, _native.DTYPE_CODE[x.dtype], 32,
                 _native.stream_ptr(x.device))
    return codes, scales


@_mxfp8_quantize_op.register_fake
def _(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    kp = (k + 31) // 32 * 32
    return (x.new_empty((m, kp), dtype=torch.uint8), x.new_empty((m, kp // 32), dtype=torch.uint8))


def mxfp8_qdq(x: torch.Tensor, group_size: int = 32) -> torch.Tensor:
    """Quantize-dequantize input to MXFP8 (E4M3 + E8M0 scales).

    Args:
        x: 2D tensor [M, K] in bf16/fp16 (CUDA)
        group_size: number of elements per scale group (32)

    Returns:
        Tensor same shape and dtype as x, with MXFP8 E4M3 quantization noise applied.
    """
    orig_dtype = x.dtype
    assert x.dim() == 2, (
        f"mxfp8_qdq only supports 2D tensors for now, but got {x.dim()}D"
    )
    assert orig_dtype in (torch.float16, torch.bfloat16), (
        f"mxfp8_qdq only supports fp16/bf16 tensors, but got {orig_dtype}"
    )
    return torch.ops.qdq_b200.mxfp8_qdq(x, group_size)


def mxfp8_quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """E4M3 codes [M, Kp] uint8 and E8M0 scales [M, Kp/32] uint8 (Kp = K rounded
    up to 32) of the same quantisation `mxfp8_qdq` applies; decoding them and
    multiplying by the scales reproduces `mxfp8_qdq(x)` exactly."""
    assert x.dim() == 2 and x.dtype in (torch.float16, torch.bfloat16)
    return torch.ops.qdq_b200.mxfp8_quantize(x)
