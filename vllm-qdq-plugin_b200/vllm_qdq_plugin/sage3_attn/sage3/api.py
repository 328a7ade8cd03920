# SPDX-License-Identifier: Apache-2.0
"""Entry points of the sm_100a Sage3 FP4 / FP8 attention.

Mirrors the reference's sage3/api.py surface:
  sageattn3_standalone(q, k, v, config, is_causal, sm_scale, per_block_mean, ...)
  sageattn3_torch_triton_standalone(..., tensor_layout="HND", quant_format, acc_dtype)
  scaled_dot_product_attention(query, key, value, attn_mask, dropout_p, is_causal, scale)
  ACC_DTYPE_MAP, ATTENTION_CONFIGS
(reference: src/vllm_qdq_plugin/sage3_attn/sage3/api.py:25-35, :394-576).

Every in-scope config runs one kernel pair in libqdq_b200.so
(`sage3_fp4_attn`, include/qdq_b200.h):
  - a pre-pass: K channel mean, per-128-token Q means, delta_s, and FP4 codes
    plus block scales of Q/K (along D) and V (along the sequence);
  - a tcgen05 flash kernel: QK^T and PV on the FP4 tensor cores, with P
    quantised in-kernel.
Config mapping:
  "mxfp4_hw"  MXFP4 with the reference hardware kernel's semantics
              (sage3/mxfp4_hw_kernel.py): E8M0 per 32, l = sum of unquantised P.
  "mxfp4"     the reference's emulated MXFP4 config (quantize.py +
              attention_kernel.py + p_quant_mxfp4) computed as the reference
              does: its fake-quantisation steps and 9-level grid {0, .5, .75,
              1, 1.5, 2, 3, 4, 6} (0.75 is no E2M1 value), held as E4M3 codes
              with E8M0 scales on kind::mxf8f6f4 MMAs; the same holds for the
              other emulated configs with E8M0 scales below.
  "nvfp4"     NVFP4 (E4M3 per 16) on real E2M1 codes: a 9-level-grid value
              times an E4M3 scale fits no block-scaled MMA operand, so parity
              with the reference's emulation is by tolerance.
  "mxfp8_hw"  MXFP8 (E4M3 + E8M0 per 32) Q/K/V and P with the reference
              hardware kernel's semantics (sage3/mxfp8_hw_kernel.py,
              quantize_to_mxfp8), on kind::mxf8f6f4 tensor-core MMAs.
  "mxfp4_s1", "mxfp8_s1"   the single-level emulated configs (P without the
              448*6 prescale); "mxfp4_s1_2level" is "mxfp4".
  "mixed_fp8qk_fp4pv", "mixed_fp4qk_fp8pv"   Q/K in one format, P/V in the
              other (emulated P of the P/V format); "*_vs" / "_vsmooth" add
              V smoothing (the V mean is subtracted before quantisation and
              added back to the output).
  "mixed_mxfp8qk_mxfp4pv_hw", "mixed_mxfp4qk_mxfp8pv_hw"   the mixed hardware
              kernels (hardware P handling, no QK smoothing).
  "mxfp4_s1_e4m3"  E2M1 with E4M3 scales per 32 (Q/K/V and single-level
              P), run on the NVFP4 block16 MMA with each scale in both of its
              16-element slots.
The kernels read the NHD or HND strides they are given; no transposing copies.
"""

from __future__ import annotations

import math
import os
import warnings
from typing import Optional, Union

import torch

from ... import _native

ACC_DTYPE_MAP = {
    # name: (qk dot, pv dot, softmax) accumulator dtypes of the reference
    "fp32": ("fp32", "fp32", "fp32"),
    "fp16_pv_only": ("fp32", "fp16", "fp32"),
    "bf16_pv_only": ("fp32", "bf16", "fp32"),
    "fp16_qk_only": ("fp16", "fp32", "fp32"),
    "bf16_qk_only": ("bf16", "fp32", "fp32"),
    "fp16_both_dot": ("fp16", "fp16", "fp32"),
    "bf16_both_dot": ("bf16", "bf16", "fp32"),
    "fp16_full": ("fp16", "fp16", "fp16"),
    "bf16_full": ("bf16", "bf16", "bf16"),
}

# config name -> quant_format of sage3_fp4_attn (include/qdq_b200.h):
#   0 mxfp4_hw, 1 nvfp4, 2 mxfp4 (two-level emulated P), 3 mxfp8_hw, 4 mxfp4_s1,
#   5 mxfp8_s1, 6 mixed_fp8qk_fp4pv, 7 mixed_fp4qk_fp8pv, 8 mixed_mxfp8qk_mxfp4pv_hw,
#   9 mixed_mxfp4qk_mxfp8pv_hw
# (reference: sage3/quant_config.py:161-330 and the hardware branches of sage3/api.py).
ATTENTION_CONFIGS: dict[str, int] = {
    "mxfp4_hw": 0, "nvfp4": 1, "mxfp4": 2, "mxfp4_s1_2level": 2, "mxfp8_hw": 3,
    "mxfp4_s1": 4, "mxfp8_s1": 5, "mixed_fp8qk_fp4pv": 6, "mixed_fp4qk_fp8pv": 7,
    "mixed_mxfp8qk_mxfp4pv_hw": 8, "mixed_mxfp4qk_mxfp8pv_hw": 9,
    "mxfp4_s1_vsmooth": 4, "mixed_fp8qk_fp4pv_vs": 6, "mixed_fp4qk_fp8pv_vs": 7, "mxfp4_s1_e4m3": 10,
}
# V smoothing (transforms.py v_smoothing: V mean subtracted before quantisation,
# added back to the output).
_VSMOOTH_CONFIGS = {"mxfp4_s1_vsmooth", "mixed_fp8qk_fp4pv_vs", "mixed_fp4qk_fp8pv_vs"}
# The mixed hardware kernels run without QK smoothing (sage3/api.py:209-291).
_NO_QK_SMOOTHING = {"mixed_mxfp8qk_mxfp4pv_hw", "mixed_mxfp4qk_mxfp8pv_hw"}

# Every config name the reference registers (sage3/quant_config.py).
REFERENCE_CONFIG_NAMES = (
    "nvfp4", "mxfp4", "mxfp4_s1", "mxfp8_s1", "mxfp4_s1_2level", "mxfp4_s1_e4m3",
    "mixed_fp8qk_fp4pv", "mixed_fp4qk_fp8pv", "mxfp4_s1_vsmooth", "mixed_fp8qk_fp4pv_vs",
    "mixed_fp4qk_fp8pv_vs", "mxfp8_hw", "mxfp4_hw", "mixed_mxfp8qk_mxfp4pv_hw", "mixed_mxfp4qk_mxfp8pv_hw")
# Names the reference registers that this build has no kernel for.
_OTHER_REFERENCE_CONFIGS = tuple(n for n in REFERENCE_CONFIG_NAMES if n not in ATTENTION_CONFIGS)

_BUILT_FORMATS = tuple(range(11))  # variants with a kernel in this build


def _get_env_bool(name: str, default: str = "0") -> bool:
    return os.getenv(name, default).lower() in ("1", "true")


def _resolve_config(config: str) -> int:
    if config not in ATTENTION_CONFIGS:
        if config in _OTHER_REFERENCE_CONFIGS:
            raise NotImplementedError(
                f"sage3 config '{config}' is not part of this build's FP4 attention "
                f"(available: {list(ATTENTION_CONFIGS)})")
        raise ValueError(f"Unknown config '{config}'. Available: {list(ATTENTION_CONFIGS.keys())}")
    fmt = ATTENTION_CONFIGS[config]
    if fmt not in _BUILT_FORMATS:
        raise NotImplementedError(f"sage3 config '{config}' has no sm_100a kernel in this build yet")
    return fmt


def _smoothing_flags(config: str, per_block_mean: bool) -> int:
    """sage3_fp4_attn's `smoothing`: bit 0 QK smoothing, bit 1 V smoothing."""
    qk = per_block_mean and not _get_env_bool("SAGE3_DISABLE_PER_BLOCK_MEAN") and config not in _NO_QK_SMOOTHING
    return int(qk) | (2 if config in _VSMOOTH_CONFIGS else 0)


@torch.library.custom_op("qdq_b200::sage3_attn", mutates_args=())
def _sage3_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout_nhd: bool, sm_scale: float,
              quant_format: int, acc_mode: int, causal: bool, smoothing: int) -> torch.Tensor:
    _native.require_cuda(q, k, v)
    out = torch.empty_like(q)
    if layout_nhd:  # [B, L, H, D]
        b_, l_, h_, d_ = q.shape
        dims = (0, 1, 2)
    else:           # [B, H, L, D]
        b_, h_, l_, d_ = q.shape
        dims = (0, 2, 1)
    strides = []
    for t in (q, k, v, out):
        strides += [t.stride(dims[0]), t.stride(dims[1]), t.stride(dims[2])]
    lib = _native.lib()
    ws = torch.empty((lib.sage3_attn_workspace_bytes(b_, l_, h_, d_),), dtype=torch.uint8,
                     device=q.device)
    import ctypes
    arr = (ctypes.c_int64 * 12)(*strides)
    _native.call("sage3_fp4_attn", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b_, l_,
                 h_, d_, arr, float(sm_scale), quant_format, acc_mode, int(causal), int(smoothing),
                 1 if q.dtype == torch.float16 else 0, ws.data_ptr(), ws.numel(), _native.stream_ptr(q.device))
    return out


@_sage3_op.register_fake
def _(q, k, v, layout_nhd, sm_scale, quant_format, acc_mode, causal, smoothing):
    return torch.empty_like(q)


# Head dims and input dtypes the FP4 kernels take (dims below 128 are
# zero-extended to 128 in the pre-pass; the reference's hardware kernels take
# 64 and 128, its emulated kernel any dim).  fp16 inputs are smoothed with
# fp16 roundings and give an fp16 output, as the reference's torch ops do.
SUPPORTED_HEAD_DIMS = (32, 64, 96, 128)
SUPPORTED_DTYPES = (torch.bfloat16, torch.float16)


def unsupported_reason(q: torch.Tensor) -> Optional[str]:
    """Why the FP4 kernels cannot take this query tensor, or None if they can."""
    if q.shape[-1] not in SUPPORTED_HEAD_DIMS:
        return f"head_dim {q.shape[-1]} (kernels take {list(SUPPORTED_HEAD_DIMS)})"
    if q.dtype not in SUPPORTED_DTYPES:
        return f"{q.dtype} inputs (kernels take {[str(d) for d in SUPPORTED_DTYPES]})"
    return None


def _check_inputs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, seq_dim: int) -> None:
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q/k/v must share one 4-D shape, got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q/k/v must share one dtype, got {q.dtype}, {k.dtype}, {v.dtype}")
    why = unsupported_reason(q)
    if why is not None:
        raise NotImplementedError(f"this build's FP4 attention does not take {why}")


_ACC_WARNED: set[str] = set()


def _acc_mode(acc_dtype: str) -> int:
    """Validate acc_dtype (the reference's ACC_DTYPE_MAP names).  The kernels
    accumulate QK^T, the softmax and PV in fp32 for every mode; the reference's
    reduced-precision modes (e.g. bf16_pv_only: O rescaled and accumulated in
    bf16, attention_kernel.py:88,169,191) are not emulated, which changes the
    output by far less than the FP4 quantisation itself.  A non-fp32 mode is
    logged once."""
    if acc_dtype not in ACC_DTYPE_MAP:
        raise ValueError(f"Unknown acc_dtype '{acc_dtype}'. Available: {list(ACC_DTYPE_MAP.keys())}")
    if acc_dtype != "fp32" and acc_dtype not in _ACC_WARNED:
        _ACC_WARNED.add(acc_dtype)
        from ..._log import init_logger
        init_logger(__name__).warning(
            "SAGE3_ACC_DTYPE=%s: this build accumulates in fp32 for every acc_dtype "
            "(the reference's %s accumulators are not emulated)", acc_dtype, ACC_DTYPE_MAP[acc_dtype])
    return 0 if acc_dtype == "fp32" else 1


def sage3_attention_nhd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, config: str = "mxfp4",
                        is_causal: bool = False, sm_scale: Optional[float] = None,
                        per_block_mean: bool = True, acc_dtype: str = "fp32") -> torch.Tensor:
    """Attention on NHD tensors [B, L, H, D] (the vllm-omni layout), output NHD."""
    fmt = _resolve_config(config)
    acc_mode = _acc_mode(acc_dtype)
    _check_inputs(q, k, v, 1)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    smoothing = _smoothing_flags(config, per_block_mean)
    return torch.ops.qdq_b200.sage3_attn(q, k, v, True, float(sm_scale), fmt, acc_mode,
                                         bool(is_causal), int(smoothing))


@torch.inference_mode()
def sageattn3_standalone(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    config: Union[str, object] = "mxfp4",
    is_causal: bool = False,
    sm_scale: Optional[float] = None,
    per_block_mean: bool = True,
    tile_size_q: int = 128,
    tile_size_k: int = 128,
    return_lse: bool = False,
    debug: bool = False,
    acc_dtype: str = "fp32",
) -> torch.Tensor:
    """SageAttention3 FP4 attention on HND tensors [B, H, N, D] -> [B, H, N, D].

    acc_dtype: every mode is accepted; the PV accumulator is fp32 in tensor
    memory for all of them (at least as accurate as the reduced-precision
    accumulators the reference's modes emulate).
    """
    name = config if isinstance(config, str) else getattr(config, "name", str(config))
    fmt = _resolve_config(name)
    acc_mode = _acc_mode(acc_dtype)
    if return_lse:
        raise NotImplementedError("return_lse is not yet supported by the sage3 composable implementation")
    _check_inputs(q, k, v, 2)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    smoothing = _smoothing_flags(name, per_block_mean)
    return torch.ops.qdq_b200.sage3_attn(q, k, v, False, float(sm_scale), fmt, acc_mode,
                                         bool(is_causal), int(smoothing))


@torch.inference_mode()
def sageattn3_torch_triton_standalone(q, k, v, tensor_layout: str = "HND", is_causal: bool = False,
                                      sm_scale: Optional[float] = None, per_block_mean: bool = True,
                                      tile_size_q: int = 128, tile_size_k: int = 128,
                                      return_lse: bool = False, debug: bool = False,
                                      quant_format: str = "mxfp4", acc_dtype: str = "fp32"):
    """Backward-compatible entry point (HND only, like the reference)."""
    if tensor_layout != "HND":
        raise ValueError("Only HND tensor layout is supported")
    return sageattn3_standalone(q, k, v, config=quant_format, is_causal=is_causal, sm_scale=sm_scale,
                                per_block_mean=per_block_mean, return_lse=return_lse,
                                acc_dtype=acc_dtype)


def scaled_dot_product_attention(query, key, value, attn_mask=None, dropout_p: float = 0.0,
                                 is_causal: bool = False, scale: Optional[float] = None, **kwargs):
    """SDPA-compatible wrapper (HND).  Same limits as the reference: no dropout,
    no masks, identical Q/K/V shapes.  The default format comes from
    SAGE3_QUANT_FORMAT (default 'nvfp4', as the reference's wrapper)."""
    if not query.is_cuda:
        raise RuntimeError("SageAttention3 requires CUDA tensors")
    if dropout_p > 0.0:
        warnings.warn(f"SageAttention3 doesn't support dropout_p={dropout_p}, ignoring",
                      UserWarning, stacklevel=2)
    if attn_mask is not None:
        warnings.warn("SageAttention3 doesn't support arbitrary attention masks, ignoring",
                      UserWarning, stacklevel=2)
    B, H, N, D = query.shape
    if key.shape != (B, H, N, D):
        raise ValueError(f"Key shape {key.shape} doesn't match query {query.shape}. "
                         "SageAttention3 requires identical Q/K/V shapes (no cross-attention or KV caching).")
    if value.shape != (B, H, N, D):
        raise ValueError(f"Value shape {value.shape} doesn't match query {query.shape}. "
                         "SageAttention3 requires identical Q/K/V shapes (no cross-attention or KV caching).")
    quant_format = kwargs.pop("quant_format", os.getenv("SAGE3_QUANT_FORMAT", "nvfp4").lower())
    acc_dtype = kwargs.pop("acc_dtype", os.getenv("SAGE3_ACC_DTYPE", "fp32").lower())
    out = sageattn3_torch_triton_standalone(query, key, value, tensor_layout="HND",
                                            is_causal=is_causal, sm_scale=scale,
                                            per_block_mean=not _get_env_bool("SAGE3_DISABLE_PER_BLOCK_MEAN"),
                                            quant_format=quant_format, acc_dtype=acc_dtype)
    if _get_env_bool("SAGE3_DEBUG") and (torch.isnan(out).any() or torch.isinf(out).any()):
        raise RuntimeError("SageAttention3 produced NaN/Inf outputs")
    return out
