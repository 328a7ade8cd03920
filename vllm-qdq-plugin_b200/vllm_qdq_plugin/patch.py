# SPDX-License-Identifier: Apache-2.0
"""Interception of vLLM's Marlin GEMM ops: run QDQ on the activation first.

Same surface as the reference (src/vllm_qdq_plugin/patch.py):
  _patch_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq)
  _patch_moe_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq)
  _patch_mla_kv_b_proj_dtype()
  apply_patches()
Each `_patch_*` replaces the attribute on `ops` and returns
(attr_name, original, patched) so apply_patches() can rebind modules that
imported the original by name.  The wrappers keep vLLM's positional
signatures (vllm/_custom_ops.py:1277-1297 and :2469).

What differs from the reference is underneath the hook: `mxfp4_qdq` is the
single-pass sm_100a kernel, and for dense MXFP4 layers whose raw weights were
captured the whole "QDQ + Marlin" pair can be replaced by the fused tcgen05
FP4 GEMM (VLLM_QDQ_FUSED_GEMM=1, see vllm_qdq_plugin.gemm).
"""

from __future__ import annotations

import functools
import sys

import torch

from . import envs
from ._log import init_logger

logger = init_logger(__name__)

_QDQ_DTYPES = (torch.float16, torch.bfloat16)


def _fp4_act_qdq(a: torch.Tensor, global_scale, mxfp4_qdq) -> torch.Tensor:
    """Activation QDQ in front of an FP4 (float4_e2m1f) Marlin GEMM: the
    reference's MXFP4 QDQ, or, with VLLM_QDQ_NVFP4_ACT=1 on an NVFP4 layer
    (global_scale given), NVFP4 QDQ with the activation's own global scale."""
    if (envs.VLLM_QDQ_NVFP4_ACT and global_scale is not None and a.dtype in _QDQ_DTYPES
            and a.shape[-1] % 16 == 0):
        from .qdq.nvfp4 import nvfp4_qdq
        return nvfp4_qdq(a, group_size=16)
    return mxfp4_qdq(a, group_size=32)


def _patch_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq):
    """Wrap ops.marlin_gemm so 2-D fp16/bf16 activations are QDQ'd first.

    Routing (reference patch.py:51-67): b_q_type float4_e2m1f -> MXFP4 QDQ
    (group 32); float8_e4m3fn -> MXFP8 QDQ; anything else passes through.
    With VLLM_QDQ_NVFP4_ACT=1 (this build only), float4_e2m1f layers that
    carry a global scale, i.e. NVFP4 Marlin layers, get NVFP4 QDQ instead.
    """
    original = ops.marlin_gemm

    def marlin_gemm(
        a: torch.Tensor,
        c: torch.Tensor | None,
        b_q_weight: torch.Tensor,
        b_bias: torch.Tensor | None,
        b_scales: torch.Tensor,
        a_scales: torch.Tensor | None,
        global_scale: torch.Tensor | None,
        b_zeros: torch.Tensor | None,
        g_idx: torch.Tensor | None,
        perm: torch.Tensor | None,
        workspace: torch.Tensor,
        b_q_type,
        size_m: int,
        size_n: int,
        size_k: int,
        is_k_full: bool = True,
        use_atomic_add: bool = False,
        use_fp32_reduce: bool = False,
        is_zp_float: bool = False,
    ) -> torch.Tensor:
        qdq_ok = a.dim() == 2 and a.dtype in _QDQ_DTYPES
        if qdq_ok and b_q_type == scalar_types.float4_e2m1f:
            trace_qdq("marlin_gemm", a.shape, a.dtype)
            if envs.VLLM_QDQ_FUSED_GEMM:
                from .gemm import fused_marlin_replacement
                out = fused_marlin_replacement(a, c, b_q_weight, b_bias, size_m, size_n, size_k,
                                               nvfp4_act=bool(envs.VLLM_QDQ_NVFP4_ACT and global_scale is not None))
                if out is not None:
                    return out
            a = _fp4_act_qdq(a, global_scale, mxfp4_qdq)
        elif qdq_ok and b_q_type == scalar_types.float8_e4m3fn:
            trace_qdq("marlin_gemm", a.shape, a.dtype)
            a = mxfp8_qdq(a, group_size=32)
        return original(a, c, b_q_weight, b_bias, b_scales, a_scales, global_scale, b_zeros,
                        g_idx, perm, workspace, b_q_type, size_m, size_n, size_k, is_k_full,
                        use_atomic_add, use_fp32_reduce, is_zp_float)

    ops.marlin_gemm = marlin_gemm
    return ("marlin_gemm", original, marlin_gemm)


def _patch_moe_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq):
    """Wrap ops.moe_wna16_marlin_gemm with the same activation QDQ.

    Routing (reference patch.py:139-152), checked in this order:
      VLLM_MARLIN_MOE_QDQ_MODE=FORCE_MXFP4 and 2-D input -> MXFP4 QDQ whatever
        b_q_type is (W4A4 emulation of models whose experts Marlin treats as FP4);
      b_q_type float4_e2m1f and 2-D -> MXFP4 QDQ;
      b_q_type float8_e4m3fn and 2-D -> MXFP8 QDQ.
    No activation dtype check on this path, as in the reference.
    With VLLM_QDQ_FUSED_GEMM=1, MXFP4 experts whose raw weights were captured
    (vllm_qdq_plugin.gemm.capture_moe_weights) run the grouped FP4 GEMM instead.
    """
    original = ops.moe_wna16_marlin_gemm

    def moe_wna16_marlin_gemm(
        input: torch.Tensor,
        output: torch.Tensor | None,
        b_qweight: torch.Tensor,
        b_bias: torch.Tensor | None,
        b_scales: torch.Tensor,
        a_scales: torch.Tensor | None,
        global_scale: torch.Tensor | None,
        b_qzeros: torch.Tensor | None,
        g_idx: torch.Tensor | None,
        perm: torch.Tensor | None,
        workspace: torch.Tensor,
        sorted_token_ids: torch.Tensor,
        expert_ids: torch.Tensor,
        num_tokens_past_padded: torch.Tensor,
        topk_weights: torch.Tensor,
        moe_block_size: int,
        top_k: int,
        mul_topk_weights: bool,
        b_q_type,
        size_m: int,
        size_n: int,
        size_k: int,
        is_k_full: bool,
        use_atomic_add: bool,
        use_fp32_reduce: bool,
        is_zp_float: bool,
        thread_k: int = -1,
        thread_n: int = -1,
        blocks_per_sm: int = -1,
    ) -> torch.Tensor:
        if (envs.VLLM_QDQ_FUSED_GEMM and input.dim() == 2 and b_q_type == scalar_types.float4_e2m1f
                and global_scale is None):
            from .gemm import fused_moe_marlin_replacement
            out = fused_moe_marlin_replacement(
                input, output, b_qweight, b_bias, a_scales, global_scale, sorted_token_ids, expert_ids,
                num_tokens_past_padded, topk_weights, moe_block_size, top_k, mul_topk_weights, size_m,
                size_n, size_k)
            if out is not None:
                trace_qdq("moe_wna16_marlin_gemm", input.shape, input.dtype)
                return out
        if input.dim() == 2:
            if envs.VLLM_MARLIN_MOE_QDQ_MODE == "FORCE_MXFP4":
                trace_qdq("moe_wna16_marlin_gemm", input.shape, input.dtype)
                input = mxfp4_qdq(input, group_size=32)
            elif b_q_type == scalar_types.float4_e2m1f:
                trace_qdq("moe_wna16_marlin_gemm", input.shape, input.dtype)
                input = _fp4_act_qdq(input, global_scale, mxfp4_qdq)
            elif b_q_type == scalar_types.float8_e4m3fn:
                trace_qdq("moe_wna16_marlin_gemm", input.shape, input.dtype)
                input = mxfp8_qdq(input, group_size=32)
        return original(input, output, b_qweight, b_bias, b_scales, a_scales, global_scale,
                        b_qzeros, g_idx, perm, workspace, sorted_token_ids, expert_ids,
                        num_tokens_past_padded, topk_weights, moe_block_size, top_k,
                        mul_topk_weights, b_q_type, size_m, size_n, size_k, is_k_full,
                        use_atomic_add, use_fp32_reduce, is_zp_float, thread_k, thread_n,
                        blocks_per_sm)

    ops.moe_wna16_marlin_gemm = moe_wna16_marlin_gemm
    return ("moe_wna16_marlin_gemm", original, moe_wna16_marlin_gemm)


def _patch_mla_kv_b_proj_dtype():
    """Keep MLA prefill-context activations floating point for packed weights.

    vLLM's MLACommonImpl._compute_prefill_context casts `kv_c_normed` to
    `kv_b_proj.weight.dtype`; with MXFP4 Marlin weights that dtype is int32.
    While the original runs, `kv_b_proj.forward` is wrapped to cast a
    non-float activation back to `params_dtype` (reference patch.py:190-240).
    """
    try:
        from vllm.model_executor.layers.attention.mla_attention import MLACommonImpl
    except ImportError:
        return

    original = MLACommonImpl._compute_prefill_context

    @functools.wraps(original)
    def _compute_prefill_context(self, *args, **kwargs):
        proj = self.kv_b_proj
        weight = getattr(proj, "weight", None)
        if weight is None or weight.dtype.is_floating_point or not hasattr(proj, "params_dtype"):
            return original(self, *args, **kwargs)
        compute_dtype = proj.params_dtype
        inner_forward = proj.forward

        @functools.wraps(inner_forward)
        def forward(input_, *fargs, **fkwargs):
            if not input_.dtype.is_floating_point:
                input_ = input_.to(compute_dtype)
            return inner_forward(input_, *fargs, **fkwargs)

        proj.forward = forward
        try:
            return original(self, *args, **kwargs)
        finally:
            proj.forward = inner_forward

    MLACommonImpl._compute_prefill_context = _compute_prefill_context
    logger.warning("QDQ patch applied: MLACommonImpl._compute_prefill_context "
                   "(packed-weight dtype fix for MXFP4/NVFP4)")


def _rebind_direct_imports(patches) -> None:
    """Modules that did `from vllm._custom_ops import marlin_gemm` hold the
    original object; point them at the wrapper too."""
    for mod in list(sys.modules.values()):
        for name, original, patched in patches:
            try:
                if getattr(mod, name, None) is original:
                    setattr(mod, name, patched)
            except Exception:
                pass


def apply_patches():
    """Install the QDQ wrappers on vllm._custom_ops (every vLLM process)."""
    import vllm._custom_ops as ops
    from vllm.scalar_type import scalar_types

    from .qdq.mxfp4 import mxfp4_qdq
    from .qdq.mxfp8 import mxfp8_qdq
    from .trace import trace_qdq

    _patch_mla_kv_b_proj_dtype()
    if envs.VLLM_QDQ_FUSED_GEMM:
        from . import gemm
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
        before = {name: getattr(mu, name, None) for name in
                  ("prepare_fp4_layer_for_marlin", "prepare_moe_fp4_layer_for_marlin",
                   "prepare_moe_mxfp4_layer_for_marlin")}
        gemm.capture_marlin_weights()
        gemm.capture_moe_weights()
        # modules that imported a preparation function by name keep the original
        _rebind_direct_imports([(name, orig, getattr(mu, name)) for name, orig in before.items()
                                if orig is not None and getattr(mu, name) is not orig])
    patches = [
        _patch_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq),
        _patch_moe_marlin_gemm(ops, scalar_types, mxfp4_qdq, mxfp8_qdq, trace_qdq),
    ]
    _rebind_direct_imports(patches)
    logger.warning("QDQ patches applied: %s (MXFP4, MXFP8)",
                   ", ".join(name for name, _, _ in patches))
