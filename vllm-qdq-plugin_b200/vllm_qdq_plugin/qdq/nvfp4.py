# SPDX-License-Identifier: Apache-2.0
"""NVFP4 activation quant-dequant on B200 (sm_100a).

The reference plugin has no NVFP4 QDQ of its own; its semantics are those of
vLLM 0.22's `ref_nvfp4_quant_dequant` (CPU branch,
vllm/model_executor/layers/quantization/utils/nvfp4_emulation_utils.py:439-478):
E2M1 elements, one E4M3 scale per 16 elements, an fp32 per-tensor global
scale `gs` in vLLM's multiplier convention (448*6/amax).  Outputs are
bit-identical to that function.

`global_scale=None` computes gs = 2688 / amax(|x|) on the device first (one
extra read of x, no host synchronisation).
"""

from __future__ import annotations

import torch

from .. import _native

AMAX_WORKSPACE_BYTES = 16


def _rows(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def _ld(x: torch.Tensor) -> int:
    return x.stride(0) if x.shape[0] > 1 else x.shape[1]


@torch.library.custom_op("qdq_b200::nvfp4_global_scale", mutates_args=())
def _nvfp4_global_scale_op(x: torch.Tensor) -> torch.Tensor:
    _native.require_cuda(x)
    x = _rows(x)
    m, k = x.shape
    gs = torch.empty((1,), dtype=torch.float32, device=x.device)
    ws = torch.empty((AMAX_WORKSPACE_BYTES // 4,), dtype=torch.int32, device=x.device)
    _native.call("qdq_nvfp4_global_scale", x.data_ptr(), gs.data_ptr(), ws.data_ptr(), m, k,
                 _ld(x), _native.DTYPE_CODE[x.dtype], _native.stream_ptr(x.device))
    return gs


@_nvfp4_global_scale_op.register_fake
def _(x: torch.Tensor) -> torch.Tensor:
    return x.new_empty((1,), dtype=torch.float32)


@torch.library.custom_op("qdq_b200::nvfp4_qdq", mutates_args=())
def _nvfp4_qdq_op(x: torch.Tensor, global_scale: torch.Tensor) -> torch.Tensor:
    _native.require_cuda(x, global_scale)
    x = _rows(x)
    m, k = x.shape
    gs = global_scale.reshape(-1)[:1].to(torch.float32)
    y = torch.empty((m, k), dtype=x.dtype, device=x.device)
    _native.call("qdq_nvfp4", x.data_ptr(), y.data_ptr(), None, None, gs.data_ptr(), m, k,
                 _ld(x), k, _native.DTYPE_CODE[x.dtype], _native.stream_ptr(x.device))
    return y


@_nvfp4_qdq_op.register_fake
def _(x: torch.Tensor, global_scale: torch.Tensor) -> torch.Tensor:
    return torch.empty_like(x, memory_format=torch.contiguous_format)


@torch.library.custom_op("qdq_b200::nvfp4_quantize", mutates_args=())
def _nvfp4_quantize_op(x: torch.Tensor, global_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    _native.require_cuda(x, global_scale)
    x = _rows(x)
    m, k = x.shape
    gs = global_scale.reshape(-1)[:1].to(torch.float32)
    codes = torch.empty((m, k // 2), dtype=torch.uint8, device=x.device)
    scales = torch.empty((m, k // 16), dtype=torch.uint8, device=x.device)
    _native.call("qdq_nvfp4", x.data_ptr(), None, codes.data_ptr(), scales.data_ptr(),
                 gs.data_ptr(), m, k, _ld(x), k, _native.DTYPE_CODE[x.dtype],
                 _native.stream_ptr(x.device))
    return codes, scales


@_nvfp4_quantize_op.register_fake
def _(x: torch.Tensor, global_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    m, k = x.shape
    return (x.new_empty((m, k // 2), dtype=torch.uint8),
            x.new_empty((m, k // 16), dtype=torch.uint8))


def _check(x: torch.Tensor, group_size: int) -> None:
    assert x.dim() == 2, f"nvfp4_qdq only supports 2D tensors, but got {x.dim()}D"
    assert x.dtype in (torch.float16, torch.bfloat16), (
        f"nvfp4_qdq only supports fp16/bf16 tensors, but got {x.dtype}")
    assert group_size == 16, f"NVFP4 uses 16-element groups, got group_size={group_size}"
    assert x.shape[1] % group_size == 0, (
        f"Weight shape K={x.shape[1]} is not divisible by block_size={group_size}")


def nvfp4_global_scale(x: torch.Tensor) -> torch.Tensor:
    """gs = 448*6 / amax(|x|) as a 1-element fp32 CUDA tensor."""
    assert x.dim() == 2 and x.dtype in (torch.float16, torch.bfloat16)
    return torch.ops.qdq_b200.nvfp4_global_scale(x)


def nvfp4_qdq(x: torch.Tensor, group_size: int = 16,
              global_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Quantize-dequantize input to NVFP4 (E2M1 + E4M3 scales + fp32 global scale).

    Args:
        x: 2D tensor [M, K] in bf16/fp16 (CUDA), K % 16 == 0
        group_size: 16
        global_scale: 1-element fp32 tensor (vLLM convention 448*6/amax), or
            None to compute it from x on the device.
    """
    _check(x, group_size)
    if global_scale is None:
        global_scale = nvfp4_global_scale(x)
    return torch.ops.qdq_b200.nvfp4_qdq(x, global_scale)


def nvfp4_quantize(x: torch.Tensor, global_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """NVFP4 codes [M, K/2] (packed E2M1) and E4M3 block scales [M, K/16]."""
    _check(x, 16)
    return torch.ops.qdq_b200.nvfp4_quantize(x, global_scale)
