# SPDX-License-Identifier: Apache-2.0
"""Quant-dequant of a tensor that lives in host memory, streamed by row blocks.

The reference's hook takes a device tensor (src/vllm_qdq_plugin/qdq/mxfp4.py:98);
a caller holding the activation in host memory copies it in, runs the hook and
copies the result out, one after the other.  `qdq_from_host` sends the rows
through the GPU in blocks instead (the C-ABI entry point `qdq_host_stream`):

    copy stream     H2D block c          H2D block c+1        ...
    current stream          QDQ block c          QDQ block c+1
    copy stream 2                   D2H block c          D2H block c+1

so the two PCIe directions and the kernel overlap, and the call takes about
as long as the larger of the two copies.  Every scale group lies inside one
row, so the result equals one quant-dequant of the whole tensor bit for bit;
NVFP4 needs its per-tensor global scale given, since it spans all rows.
"""

from __future__ import annotations

import math

import torch

from .. import _native

_FORMATS = {"mxfp4": 0, "nvfp4": 1, "mxfp8": 2}  # QDQ_FORMAT_* of include/qdq_b200.h


def qdq_from_host(x: torch.Tensor, fmt: str = "mxfp4", *, global_scale: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, device: torch.device | int | None = None,
                  block_bytes: int = 16 << 20, depth: int = 3, non_blocking: bool = False) -> torch.Tensor:
    """Quant-dequant the host tensor `x` [M, K] (bf16/fp16) on a GPU into host memory.

    Args:
        x: host tensor, 2-D, bf16 or fp16.  Pin it (`x.pin_memory()`) for the
            copies to overlap.
        fmt: "mxfp4" (E2M1 + E8M0 per 32), "mxfp8" (E4M3 + E8M0 per 32) or
            "nvfp4" (E2M1 + E4M3 per 16 with the fp32 global scale).
        global_scale: NVFP4 only, required: 1-element fp32 tensor in vLLM's
            multiplier convention (448*6/amax over the whole tensor).
        out: host tensor [M, K] of x's dtype for the result; allocated pinned
            if None.
        device: the GPU to run on (default: the current one).
        block_bytes: input bytes per row block (rounded down to whole rows).
            Measured on B200 over PCIe: 16 MB blocks reach about 1.6x the
            one-direction copy rate for config 2; blocks of 1-4 MB lose to
            per-copy overheads, and larger ones to pipeline fill and drain.
        depth: row blocks in flight (1..8).
        non_blocking: if False, return after the result is in `out`; if
            True, return once the work is enqueued on the current stream
            (synchronise it before reading `out`).

    Returns `out`, bit-identical to the device hook applied to `x.cuda()`.
    """
    if fmt not in _FORMATS:
        raise ValueError(f"unknown format {fmt!r}; expected one of {sorted(_FORMATS)}")
    assert x.dim() == 2, f"qdq_from_host expects a 2D tensor, got {x.dim()}D"
    assert x.dtype in (torch.float16, torch.bfloat16), (
        f"qdq_from_host only supports fp16/bf16 tensors, but got {x.dtype}")
    if x.is_cuda:
        raise ValueError("qdq_from_host takes a host tensor; call the device hook for CUDA tensors")
    if fmt == "nvfp4":
        if global_scale is None:
            raise ValueError("nvfp4 from host needs global_scale (448*6/amax over the whole tensor)")
        assert x.shape[1] % 16 == 0, f"Weight shape K={x.shape[1]} is not divisible by block_size=16"
    if not 1 <= depth <= 8 or block_bytes < 1:
        raise ValueError("depth must be in 1..8 and block_bytes positive")
    if x.stride(-1) != 1:
        x = x.contiguous()
    m, k = x.shape
    if out is None:
        out = torch.empty((m, k), dtype=x.dtype, pin_memory=True)
    elif out.shape != x.shape or out.dtype != x.dtype or out.is_cuda or out.stride(-1) != 1:
        raise ValueError("out must be a host tensor of x's shape and dtype with unit stride in K")
    if m == 0 or k == 0:
        return out

    if isinstance(device, int):
        dev = torch.device("cuda", device)
    elif device is None or torch.device(device).index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device(device)
    dtype = _native.DTYPE_CODE[x.dtype]
    row_bytes = k * x.element_size()
    # whole rows per block, a multiple of 8 / gcd(K, 8) so that every staging
    # block starts 16-byte aligned (the vectorised kernels need it)
    unit = 8 // math.gcd(k, 8)
    rows = min(m, max(unit, block_bytes // row_bytes // unit * unit))
    lib = _native.lib()
    nbytes = lib.qdq_host_stream_staging_bytes(rows, k, dtype, min(depth, -(-m // rows)))
    with torch.cuda.device(dev):
        staging = torch.empty((nbytes,), dtype=torch.uint8, device=dev)
        gs = None
        if fmt == "nvfp4":
            gs = global_scale.reshape(-1)[:1].to(device=dev, dtype=torch.float32)
        stream = torch.cuda.current_stream(dev)
        _native.call("qdq_host_stream", _FORMATS[fmt], x.data_ptr(), out.data_ptr(), _native.ptr(gs),
                     m, k, x.stride(0) if m > 1 else k, out.stride(0) if m > 1 else k, dtype,
                     staging.data_ptr(), nbytes, rows, stream.cuda_stream)
        # `staging` is freed here in the current stream's order, which the
        # library extended past its last copy
        if not non_blocking:
            stream.synchronize()
    return out
