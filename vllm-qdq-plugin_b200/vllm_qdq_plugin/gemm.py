# SPDX-License-Identifier: Apache-2.0
"""Fused MXFP4 linear: activation quantisation + tcgen05 block-scaled FP4 GEMM.

The reference simulates W4A4 by running `mxfp4_qdq` on the activation and
then vLLM's Marlin kernel (bf16 activation x dequantised FP4 weight)
(reference: src/vllm_qdq_plugin/patch.py:51-57; vllm/_custom_ops.py:1277).
A QDQ'd activation is exactly representable in MXFP4, so the same product is
computed here with FP4 tensor-core MMAs on codes + E8M0 scales
(`fp4_gemm_mxf4` / `fp4_linear_mxf4` in include/qdq_b200.h).

Marlin layers carry Marlin-repacked weights that this kernel cannot read, so
with VLLM_QDQ_FUSED_GEMM=1 `capture_marlin_weights()` records each MXFP4
layer's raw weight codes / scales / bias when vLLM prepares it for Marlin
(vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py:205
prepare_fp4_layer_for_marlin) and keys them by the repacked weight, which the
patched `marlin_gemm` receives as `b_q_weight`.  Layers without a captured
weight keep the reference path (QDQ + Marlin).
"""

from __future__ import annotations

import dataclasses
import functools
import threading

import torch

from . import _native
from ._log import init_logger
from .qdq.mxfp4 import mxfp4_quantize

logger = init_logger(__name__)


@dataclasses.dataclass
class Mxfp4Weight:
    """An MXFP4 weight [N, K] in the layout the tcgen05 GEMM reads."""

    codes: torch.Tensor     # uint8 [N, K/2], element 2j in the low nibble
    sf_tiled: torch.Tensor  # uint8, tiled E8M0 scales (qdq_sf_tile layout)
    n: int
    k: int
    bias: torch.Tensor | None = None

    @property
    def device(self) -> torch.device:
        return self.codes.device


def _tile_scales(scales: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    lib = _native.lib()
    nbytes = lib.qdq_sf_tiled_bytes(rows, k)
    out = torch.empty((nbytes,), dtype=torch.uint8, device=scales.device)
    _native.call("qdq_sf_tile", scales.data_ptr(), out.data_ptr(), rows, k, scales.stride(0), 32,
                 _native.stream_ptr(scales.device))
    return out


def prepare_mxfp4_weight(codes: torch.Tensor, scales: torch.Tensor,
                         bias: torch.Tensor | None = None) -> Mxfp4Weight:
    """codes uint8 [N, K/2] (packed E2M1), scales uint8 [N, K/32] (E8M0)."""
    _native.require_cuda(codes, scales)
    assert codes.dtype == torch.uint8 and scales.dtype == torch.uint8
    n, kh = codes.shape
    k = kh * 2
    assert k % 32 == 0 and scales.shape == (n, k // 32), (codes.shape, scales.shape)
    codes = codes.contiguous()
    scales = scales.contiguous()
    return Mxfp4Weight(codes=codes, sf_tiled=_tile_scales(scales, n, k), n=n, k=k, bias=bias)


@torch.library.custom_op("qdq_b200::mxfp4_gemm_codes", mutates_args=())
def _gemm_codes_op(a_codes: torch.Tensor, a_sf_tiled: torch.Tensor, w_codes: torch.Tensor,
                   w_sf_tiled: torch.Tensor, bias: torch.Tensor | None, out_fp16: bool) -> torch.Tensor:
    _native.require_cuda(a_codes, w_codes)
    m, n, k = a_codes.shape[0], w_codes.shape[0], w_codes.shape[1] * 2
    out = torch.empty((m, n), dtype=torch.float16 if out_fp16 else torch.bfloat16,
                      device=a_codes.device)
    _native.call("fp4_gemm_mxf4", a_codes.data_ptr(), a_sf_tiled.data_ptr(), w_codes.data_ptr(),
                 w_sf_tiled.data_ptr(), _native.ptr(bias), out.data_ptr(), m, n, k,
                 a_codes.stride(0), w_codes.stride(0), n, int(out_fp16),
                 _native.stream_ptr(a_codes.device))
    return out


@_gemm_codes_op.register_fake
def _(a_codes, a_sf_tiled, w_codes, w_sf_tiled, bias, out_fp16):
    return a_codes.new_empty((a_codes.shape[0], w_codes.shape[0]),
                             dtype=torch.float16 if out_fp16 else torch.bfloat16)


@torch.library.custom_op("qdq_b200::mxfp4_linear", mutates_args=())
def _linear_op(a: torch.Tensor, w_codes: torch.Tensor, w_sf_tiled: torch.Tensor,
               bias: torch.Tensor | None) -> torch.Tensor:
    _native.require_cuda(a, w_codes, w_sf_tiled)
    a = a if a.stride(-1) == 1 else a.contiguous()
    m, k = a.shape
    n = w_codes.shape[0]
    lib = _native.lib()
    ws = torch.empty((lib.fp4_linear_workspace_bytes(m, k),), dtype=torch.uint8, device=a.device)
    out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _native.call("fp4_linear_mxf4", a.data_ptr(), a.stride(0) if m > 1 else k,
                 _native.DTYPE_CODE[a.dtype], w_codes.data_ptr(), w_sf_tiled.data_ptr(),
                 _native.ptr(bias), out.data_ptr(), m, n, k, w_codes.stride(0), n, ws.data_ptr(),
                 ws.numel(), _native.stream_ptr(a.device))
    return out


@_linear_op.register_fake
def _(a, w_codes, w_sf_tiled, bias):
    return a.new_empty((a.shape[0], w_codes.shape[0]))


def mxfp4_linear(a: torch.Tensor, weight: Mxfp4Weight, bias: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = mxfp4_qdq(a) @ dequant(weight)^T (+ bias), fp32 accumulation.

    a: [M, K] bf16/fp16 CUDA tensor, K % 32 == 0.  Output dtype = a.dtype.
    """
    assert a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16)
    assert a.shape[1] == weight.k, (a.shape, weight.k)
    if bias is None:
        bias = weight.bias
    if bias is not None:
        bias = bias.to(a.dtype).contiguous()
    return torch.ops.qdq_b200.mxfp4_linear(a, weight.codes, weight.sf_tiled, bias)


def mxfp4_gemm_codes(a_codes: torch.Tensor, a_scales: torch.Tensor, weight: Mxfp4Weight,
                     bias: torch.Tensor | None = None, out_dtype=torch.bfloat16) -> torch.Tensor:
    """GEMM on pre-quantised activation codes [M, K/2] + row-major E8M0 scales [M, K/32]."""
    m = a_codes.shape[0]
    a_sf = _tile_scales(a_scales.contiguous(), m, weight.k)
    return torch.ops.qdq_b200.mxfp4_gemm_codes(a_codes.contiguous(), a_sf, weight.codes,
                                               weight.sf_tiled, bias, out_dtype == torch.float16)


# ---------------------------------------------------------------------------
# NVFP4 linear (E2M1 + UE4M3 per 16 + fp32 tensor scales), kind::mxf4nvf4
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class Nvfp4Weight:
    """An NVFP4 weight [N, K]: codes, E4M3 scales per 16 (tiled) and the fp32
    tensor scale that multiplies them (vLLM's `weight_global_scale`)."""

    codes: torch.Tensor     # uint8 [N, K/2], element 2j in the low nibble
    sf_tiled: torch.Tensor  # uint8, tiled E4M3 scales (qdq_sf_tile, block 16)
    global_scale: float     # dequantised weight = code * scale * global_scale
    n: int
    k: int
    bias: torch.Tensor | None = None


def prepare_nvfp4_weight(codes: torch.Tensor, scales: torch.Tensor, global_scale: float,
                         bias: torch.Tensor | None = None) -> Nvfp4Weight:
    """codes uint8 [N, K/2] (packed E2M1); scales [N, K/16] E4M3 (uint8 or
    float8_e4m3fn); global_scale: the weight's fp32 tensor scale."""
    _native.require_cuda(codes, scales)
    codes = codes.view(torch.uint8).contiguous()
    scales = scales.view(torch.uint8).contiguous()
    n, kh = codes.shape
    k = kh * 2
    assert k % 32 == 0 and scales.shape == (n, k // 16), (codes.shape, scales.shape)
    lib = _native.lib()
    sf = torch.empty((lib.qdq_sf16_tiled_bytes(n, k),), dtype=torch.uint8, device=codes.device)
    _native.call("qdq_sf_tile", scales.data_ptr(), sf.data_ptr(), n, k, scales.stride(0), 16,
                 _native.stream_ptr(codes.device))
    return Nvfp4Weight(codes=codes, sf_tiled=sf, global_scale=float(global_scale), n=n, k=k, bias=bias)


@torch.library.custom_op("qdq_b200::nvfp4_linear", mutates_args=())
def _nvfp4_linear_op(a: torch.Tensor, w_codes: torch.Tensor, w_sf_tiled: torch.Tensor, w_global_scale: float,
                     bias: torch.Tensor | None, a_global_scale: torch.Tensor | None) -> torch.Tensor:
    _native.require_cuda(a, w_codes, w_sf_tiled)
    a = a if a.stride(-1) == 1 else a.contiguous()
    m, k = a.shape
    n = w_codes.shape[0]
    lib = _native.lib()
    ws = torch.empty((lib.fp4_linear_nvf4_workspace_bytes(m, k),), dtype=torch.uint8, device=a.device)
    out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    gs = None if a_global_scale is None else a_global_scale.reshape(-1)[:1].to(torch.float32).contiguous()
    _native.call("fp4_linear_nvf4", a.data_ptr(), a.stride(0) if m > 1 else k, _native.DTYPE_CODE[a.dtype],
                 _native.ptr(gs), w_codes.data_ptr(), w_sf_tiled.data_ptr(), float(w_global_scale),
                 _native.ptr(bias), out.data_ptr(), m, n, k, w_codes.stride(0), n, ws.data_ptr(), ws.numel(),
                 _native.stream_ptr(a.device))
    return out


@_nvfp4_linear_op.register_fake
def _(a, w_codes, w_sf_tiled, w_global_scale, bias, a_global_scale):
    return a.new_empty((a.shape[0], w_codes.shape[0]))


def nvfp4_linear(a: torch.Tensor, weight: Nvfp4Weight, bias: torch.Tensor | None = None,
                 a_global_scale: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = nvfp4(a) @ dequant(weight)^T (+ bias), fp32 accumulation.

    The activation is quantised exactly as nvfp4_qdq does (group 16, E4M3
    scales, gs_a = 2688 / amax(a) unless `a_global_scale` is given), and the
    product is formed from the codes on the FP4 tensor cores, so it equals
    nvfp4_qdq(a) @ dequant(W)^T up to nvfp4_qdq's bf16 rounding of each
    activation element and fp32 summation order.  a: [M, K] bf16/fp16 CUDA,
    K % 32 == 0.  Output dtype = a.dtype."""
    assert a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16)
    assert a.shape[1] == weight.k, (a.shape, weight.k)
    if bias is None:
        bias = weight.bias
    if bias is not None:
        bias = bias.to(a.dtype).contiguous()
    return torch.ops.qdq_b200.nvfp4_linear(a, weight.codes, weight.sf_tiled, weight.global_scale, bias,
                                           a_global_scale)


# ---------------------------------------------------------------------------
# Marlin-layer capture (VLLM_QDQ_FUSED_GEMM=1)
# ---------------------------------------------------------------------------
_REGISTRY: dict[int, Mxfp4Weight | Nvfp4Weight] = {}
_REG_LOCK = threading.Lock()


def register_marlin_weight(marlin_weight: torch.Tensor, weight: Mxfp4Weight | Nvfp4Weight) -> None:
    with _REG_LOCK:
        _REGISTRY[marlin_weight.data_ptr()] = weight


def lookup_marlin_weight(marlin_weight: torch.Tensor) -> Mxfp4Weight | Nvfp4Weight | None:
    return _REGISTRY.get(marlin_weight.data_ptr())


def fused_marlin_replacement(a, c, b_q_weight, b_bias, size_m, size_n, size_k, nvfp4_act: bool = False):
    """Run the fused FP4 linear for a captured layer; None means "keep the
    reference path" (QDQ + Marlin).  MXFP4 layers take the MXFP4 linear (the
    reference's MXFP4 activation QDQ, fused).  NVFP4 layers take the NVFP4
    linear only with nvfp4_act (VLLM_QDQ_NVFP4_ACT=1): the reference itself
    applies MXFP4 QDQ to their activations, which no NVFP4 MMA can take."""
    w = lookup_marlin_weight(b_q_weight)
    if w is None or a.shape[1] != w.k or w.n != size_n or size_k != w.k:
        return None
    bias = w.bias if b_bias is not None else None
    if isinstance(w, Nvfp4Weight):
        if not nvfp4_act or a.shape[1] % 32 != 0:
            return None
        out = nvfp4_linear(a, w, bias)
    else:
        out = mxfp4_linear(a, w, bias)
    if c is not None:
        c.copy_(out)
        return c
    return out


def capture_marlin_weights() -> bool:
    """Wrap vLLM's prepare_fp4_layer_for_marlin to keep the raw MXFP4 weights."""
    try:
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
    except ImportError:
        return False
    original = mu.prepare_fp4_layer_for_marlin
    if getattr(original, "_qdq_b200_capture", False):
        return True

    @functools.wraps(original)
    def prepare_fp4_layer_for_marlin(layer, input_dtype=None):
        raw = None
        if input_dtype is None or input_dtype.itemsize != 1:
            bias = getattr(layer, "bias", None)
            gs = getattr(layer, "weight_global_scale", None)
            raw = (layer.weight.data, layer.weight_scale.data,
                   None if bias is None else bias.data.clone(),
                   None if gs is None else float(gs.data.reshape(-1)[0].float()))
        result = original(layer, input_dtype)
        if raw is not None and raw[0].is_cuda:
            codes, scales, bias, gs = raw
            if gs is None:   # MXFP4: E8M0 scales per 32
                w = prepare_mxfp4_weight(codes.view(torch.uint8), scales.view(torch.uint8), bias)
            else:            # NVFP4: E4M3 scales per 16 and the weight's tensor scale
                w = prepare_nvfp4_weight(codes.view(torch.uint8), scales.view(torch.uint8), gs, bias)
            register_marlin_weight(layer.weight, w)
        return result

    prepare_fp4_layer_for_marlin._qdq_b200_capture = True
    mu.prepare_fp4_layer_for_marlin = prepare_fp4_layer_for_marlin
    logger.warning("vllm-qdq-plugin: capturing raw MXFP4 / NVFP4 weights for the fused FP4 GEMM")
    return True


# ---------------------------------------------------------------------------
# Grouped MXFP4 MoE GEMM (replaces QDQ + moe_wna16_marlin_gemm for MXFP4 experts)
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class Mxfp4MoeWeight:
    """MXFP4 expert weights [E, N, K] in the layout the grouped tcgen05 GEMM reads."""

    codes: torch.Tensor     # uint8 [E, N, K/2], element 2j in the low nibble
    sf_tiled: torch.Tensor  # uint8 [E * qdq_sf_tiled_bytes(N, K)], per-expert tiled E8M0 scales
    e: int
    n: int
    k: int


def prepare_mxfp4_moe_weight(codes: torch.Tensor, scales: torch.Tensor) -> Mxfp4MoeWeight:
    """codes uint8 [E, N, K/2] (packed E2M1), scales uint8 [E, N, K/32] (E8M0)."""
    _native.require_cuda(codes, scales)
    codes = codes.view(torch.uint8).contiguous()
    scales = scales.view(torch.uint8).contiguous()
    e, n, kh = codes.shape
    k = kh * 2
    assert k % 32 == 0 and scales.shape == (e, n, k // 32), (codes.shape, scales.shape)
    per = _native.lib().qdq_sf_tiled_bytes(n, k)
    sf = torch.empty((e * per,), dtype=torch.uint8, device=codes.device)
    sp = _native.stream_ptr(codes.device)
    for i in range(e):
        _native.call("qdq_sf_tile", scales[i].data_ptr(), sf[i * per:].data_ptr(), n, k, scales.stride(1), 32, sp)
    return Mxfp4MoeWeight(codes=codes, sf_tiled=sf, e=e, n=n, k=k)


@torch.library.custom_op("qdq_b200::mxfp4_moe_linear", mutates_args=("out",))
def _moe_op(a: torch.Tensor, w_codes: torch.Tensor, w_sf_tiled: torch.Tensor, sorted_token_ids: torch.Tensor,
            expert_ids: torch.Tensor, num_tokens_post_padded: torch.Tensor, topk_weights: torch.Tensor | None,
            moe_block_size: int, top_k: int, mul_topk_weights: bool, out: torch.Tensor) -> None:
    _native.require_cuda(a, w_codes, w_sf_tiled, sorted_token_ids, expert_ids, num_tokens_post_padded, out)
    a = a if a.stride(-1) == 1 else a.contiguous()
    e, n, kh = w_codes.shape
    lib = _native.lib()
    ws = torch.empty((lib.fp4_moe_workspace_bytes(sorted_token_ids.numel(), moe_block_size, kh * 2),),
                     dtype=torch.uint8, device=a.device)
    _native.call("fp4_moe_mxf4", a.data_ptr(), a.stride(0) if a.shape[0] > 1 else a.shape[1],
                 _native.DTYPE_CODE[a.dtype], w_codes.data_ptr(), w_sf_tiled.data_ptr(), e,
                 sorted_token_ids.data_ptr(), expert_ids.data_ptr(), num_tokens_post_padded.data_ptr(),
                 _native.ptr(topk_weights), sorted_token_ids.numel(), moe_block_size, top_k,
                 int(mul_topk_weights), out.data_ptr(), out.stride(0), a.shape[0], n, kh * 2,
                 ws.data_ptr(), ws.numel(), _native.stream_ptr(a.device))


@_moe_op.register_fake
def _(a, w_codes, w_sf_tiled, sorted_token_ids, expert_ids, num_tokens_post_padded, topk_weights,
      moe_block_size, top_k, mul_topk_weights, out):
    return None


def mxfp4_moe_linear(a: torch.Tensor, weight: Mxfp4MoeWeight, sorted_token_ids: torch.Tensor,
                     expert_ids: torch.Tensor, num_tokens_post_padded: torch.Tensor,
                     topk_weights: torch.Tensor | None, moe_block_size: int, top_k: int,
                     mul_topk_weights: bool, out: torch.Tensor | None = None) -> torch.Tensor:
    """For every routed slot s (vLLM's moe_align_block_size layout):
    out[s] = mxfp4_qdq(a[s // top_k]) @ dequant(W[expert of s's block])^T (x topk_weights[s]).

    a: [M, K] bf16/fp16; out: [M * top_k, N] (allocated when None; rows of
    slots that are not routed keep their contents)."""
    assert a.dim() == 2 and a.dtype in (torch.bfloat16, torch.float16) and a.shape[1] == weight.k
    assert sorted_token_ids.dtype == torch.int32 and expert_ids.dtype == torch.int32
    if out is None:
        out = torch.empty((a.shape[0] * top_k, weight.n), dtype=a.dtype, device=a.device)
    tw = topk_weights.reshape(-1).float().contiguous() if topk_weights is not None else None
    torch.ops.qdq_b200.mxfp4_moe_linear(a, weight.codes, weight.sf_tiled, sorted_token_ids, expert_ids,
                                        num_tokens_post_padded, tw, moe_block_size, top_k,
                                        bool(mul_topk_weights), out)
    return out


_MOE_REGISTRY: dict[int, Mxfp4MoeWeight] = {}


def register_marlin_moe_weight(marlin_weight: torch.Tensor, weight: Mxfp4MoeWeight) -> None:
    with _REG_LOCK:
        _MOE_REGISTRY[marlin_weight.data_ptr()] = weight


def fused_moe_marlin_replacement(input, output, b_qweight, b_bias, a_scales, global_scale, sorted_token_ids,
                                 expert_ids, num_tokens_past_padded, topk_weights, moe_block_size, top_k,
                                 mul_topk_weights, size_m, size_n, size_k):
    """The grouped FP4 GEMM for a captured MXFP4 MoE layer; None means "keep
    the reference path" (not captured, bias, NVFP4 global scale, 8-bit input)."""
    w = _MOE_REGISTRY.get(b_qweight.data_ptr())
    if (w is None or b_bias is not None or a_scales is not None or global_scale is not None
            or input.dim() != 2 or input.dtype not in (torch.bfloat16, torch.float16)
            or tuple(input.shape) != (size_m, size_k) or w.n != size_n or w.k != size_k
            or not 1 <= moe_block_size <= 64 or sorted_token_ids.dtype != torch.int32
            or expert_ids.dtype != torch.int32):
        return None
    return mxfp4_moe_linear(input, w, sorted_token_ids, expert_ids, num_tokens_past_padded, topk_weights,
                            moe_block_size, top_k, mul_topk_weights, output)


def capture_moe_weights() -> bool:
    """Wrap vLLM's MXFP4 MoE Marlin preparation (in-place and pure variants,
    marlin_utils_fp4.py prepare_moe_fp4_layer_for_marlin /
    prepare_moe_mxfp4_layer_for_marlin) to keep each layer's raw expert weights."""
    try:
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
    except ImportError:
        return False

    def keep(marlin_w13, marlin_w2, w13, w13_scale, w2, w2_scale):
        if w13.is_cuda:
            register_marlin_moe_weight(marlin_w13, prepare_mxfp4_moe_weight(w13, w13_scale))
            register_marlin_moe_weight(marlin_w2, prepare_mxfp4_moe_weight(w2, w2_scale))

    original = getattr(mu, "prepare_moe_fp4_layer_for_marlin", None)
    if original is not None and not getattr(original, "_qdq_b200_capture", False):
        @functools.wraps(original)
        def prepare_moe_fp4_layer_for_marlin(layer, input_dtype=None):
            raw = None
            if not hasattr(layer, "w13_weight_scale_2") and (input_dtype is None or input_dtype.itemsize != 1):
                raw = (layer.w13_weight.data, layer.w13_weight_scale.data, layer.w2_weight.data,
                       layer.w2_weight_scale.data)
            result = original(layer, input_dtype)
            if raw is not None:
                keep(layer.w13_weight, layer.w2_weight, *raw)
            return result

        prepare_moe_fp4_layer_for_marlin._qdq_b200_capture = True
        mu.prepare_moe_fp4_layer_for_marlin = prepare_moe_fp4_layer_for_marlin

    pure = getattr(mu, "prepare_moe_mxfp4_layer_for_marlin", None)
    if pure is not None and not getattr(pure, "_qdq_b200_capture", False):
        @functools.wraps(pure)
        def prepare_moe_mxfp4_layer_for_marlin(layer, w13, w2, w13_scale, w2_scale, w13_bias, w2_bias):
            result = pure(layer, w13, w2, w13_scale, w2_scale, w13_bias, w2_bias)
            input_dtype = mu.get_marlin_input_dtype()
            if input_dtype is None or input_dtype.itemsize != 1:
                keep(result[0], result[1], w13, w13_scale, w2, w2_scale)
            return result

        prepare_moe_mxfp4_layer_for_marlin._qdq_b200_capture = True
        mu.prepare_moe_mxfp4_layer_for_marlin = prepare_moe_mxfp4_layer_for_marlin
    logger.warning("vllm-qdq-plugin: capturing raw MXFP4 MoE weights for the grouped FP4 GEMM")
    return True
