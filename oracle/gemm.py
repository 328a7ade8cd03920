"""CPU oracle of "MXFP4 QDQ + Marlin GEMM" (the reference's dense FP4 linear).

TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py baselines).

The reference path is `mxfp4_qdq(a)` (src/vllm_qdq_plugin/patch.py:57) followed
by vLLM's `marlin_gemm` (vllm/_custom_ops.py:1277), which multiplies the bf16
activation by the dequantised MXFP4 weight (E2M1 value x 2^(e8m0-127)) with
fp32 accumulation and rounds to the activation dtype.  Marlin itself is a
compiled kernel that is not restated here; its products are exact, so the
oracle forms them exactly (float64) and the tests allow bf16 output rounding
plus an fp32-accumulation bound.  The E2M1 table and E8M0 power-of-two scale
follow the reference's own dequantiser
(src/vllm_qdq_plugin/sage3_attn/sage3/mxfp4_hw_kernel.py:31-35, :64-70, :119-139).
"""

from __future__ import annotations

import numpy as np

from . import qdq as oq

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def dequant_mxfp4(codes: np.ndarray, scales: np.ndarray, block: int = 32) -> np.ndarray:
    """codes uint8 [R, K/2] (element 2j in the low nibble), scales uint8 E8M0 [R, K/block]."""
    lo = E2M1[codes & 0xF]
    hi = E2M1[codes >> 4]
    vals = np.stack([lo, hi], axis=-1).reshape(codes.shape[0], -1)
    sc = np.exp2(scales.astype(np.float64) - 127.0)
    return vals * np.repeat(sc, block, axis=1)[:, : vals.shape[1]]


def bf16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def qdq_linear_exact(a_bits: np.ndarray, w_codes: np.ndarray, w_scales: np.ndarray,
                     bias: np.ndarray | None = None, fp16: bool = False):
    """Exact (float64) mxfp4_qdq(a) @ dequant(W)^T (+ bias) and the per-output sum
    of |products| (bound for fp32-accumulation error)."""
    aq = oq.mxfp4_qdq(a_bits, fp16=fp16)
    if fp16:
        a = aq.view(np.float16).astype(np.float64)
    else:
        a = bf16_bits_to_f64(aq)
    w = dequant_mxfp4(w_codes, w_scales)
    out = a @ w.T
    absum = np.abs(a) @ np.abs(w).T
    if bias is not None:
        out = out + bias.astype(np.float64)[None, :]
    return out, absum


def random_mxfp4_weight(n: int, k: int, seed: int, exp_lo: int = -10, exp_hi: int = -4):
    """Config-3 weights: uniform random E2M1 nibbles, E8M0 exponents in [exp_lo, exp_hi]."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = (127 + rng.integers(exp_lo, exp_hi + 1, size=(n, k // 32))).astype(np.uint8)
    return codes, scales


def moe_align(topk_ids: np.ndarray, num_experts: int, block: int):
    """vLLM's moe_align_block_size layout (vllm/model_executor/layers/fused_moe/
    moe_align_block_size.py): the M*top_k token slots (slot = token * top_k + j)
    grouped by expert in slot order, each expert's run padded to a multiple of
    `block` with the sentinel M*top_k.  Returns int32 sorted_token_ids,
    expert_ids (one per block) and num_tokens_post_padded [1]."""
    m, top_k = topk_ids.shape
    flat = topk_ids.reshape(-1)
    sorted_ids, experts = [], []
    for e in range(num_experts):
        slots = np.nonzero(flat == e)[0]
        if len(slots) == 0:
            continue
        pad = (-len(slots)) % block
        sorted_ids.extend(slots.tolist() + [m * top_k] * pad)
        experts.extend([e] * ((len(slots) + pad) // block))
    return (np.array(sorted_ids, np.int32), np.array(experts, np.int32),
            np.array([len(sorted_ids)], np.int32))


def moe_linear_exact(a_bits: np.ndarray, w_codes: np.ndarray, w_scales: np.ndarray,
                     sorted_ids: np.ndarray, expert_ids: np.ndarray, num_post_padded: int, block: int,
                     top_k: int, topk_weights: np.ndarray | None = None, fp16: bool = False):
    """Exact (float64) grouped MoE linear, the reference's "mxfp4_qdq(input),
    then moe_wna16_marlin_gemm" (src/vllm_qdq_plugin/patch.py:139-152): for each
    routed slot s of a block with expert e, out[s] = mxfp4_qdq(a[s // top_k]) .
    dequant(W_e)^T (x topk_weights[s]).  Returns {slot: (row, absum row)}."""
    m = a_bits.shape[0]
    rows = {}
    for b in range(num_post_padded // block):
        e = int(expert_ids[b])
        if e < 0:
            continue
        slots = [int(s) for s in sorted_ids[b * block:(b + 1) * block] if 0 <= s < m * top_k]
        if not slots:
            continue
        tok = np.array([s // top_k for s in slots])
        out, absum = qdq_linear_exact(a_bits[tok], w_codes[e], w_scales[e], fp16=fp16)
        for i, s in enumerate(slots):
            wgt = 1.0 if topk_weights is None else float(np.float32(topk_weights[s]))
            rows[s] = (out[i] * wgt, absum[i] * abs(wgt))
    return rows


def e4m3_values(b: np.ndarray) -> np.ndarray:
    """float64 value of E4M3 (float8_e4m3fn) bytes."""
    b = np.asarray(b, np.uint8).astype(np.int64)
    exp, man = (b >> 3) & 0xF, b & 7
    mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1 + man / 8.0) * np.exp2(exp - 7.0))
    mag = np.where((exp == 15) & (man == 7), np.nan, mag)
    return np.where(b & 0x80, -mag, mag)


def dequant_nvfp4(codes: np.ndarray, scales: np.ndarray, global_scale: float) -> np.ndarray:
    """NVFP4 weight [R, K]: E2M1 code x E4M3 scale (per 16) x the fp32 tensor
    scale, vLLM's convention for NVFP4 layers (marlin_utils_fp4.py
    rand_marlin_weight_nvfp4_like: weight_ref = fp4 * global_scale * scales)."""
    lo = E2M1[codes & 0xF]
    hi = E2M1[codes >> 4]
    vals = np.stack([lo, hi], axis=-1).reshape(codes.shape[0], -1)
    return vals * np.repeat(e4m3_values(scales), 16, axis=1) * float(global_scale)


def nvfp4_linear_exact(a_bits: np.ndarray, w_codes: np.ndarray, w_scales: np.ndarray, w_global_scale: float,
                       fp16: bool = False, a_global_scale: float | None = None):
    """The NVFP4 linear with NVFP4 activations, exactly (float64):
      exact     nvfp4(a) @ W^T with the activation dequantised as code * s / gs_a
                before any rounding (what the block16 tensor-core GEMM computes);
      via_qdq   nvfp4_qdq(a) @ W^T, the activation rounded to bf16/fp16 first
                (what nvfp4_qdq + Marlin computes);
      absum     sum |a_k w_k| per output (bound for fp32-accumulation error).
    gs_a = 2688 / amax(a) (vLLM's ref_nvfp4_quant_dequant convention) unless given."""
    gs = oq.nvfp4_global_scale(a_bits, fp16=fp16) if a_global_scale is None else a_global_scale
    y, codes, scales = oq.nvfp4_qdq(a_bits, gs, fp16=fp16, codes=True)
    lo, hi = E2M1[codes & 0xF], E2M1[codes >> 4]
    a_codes = np.stack([lo, hi], axis=-1).reshape(codes.shape[0], -1)
    a_exact = a_codes * np.repeat(e4m3_values(scales), 16, axis=1) / np.float64(np.float32(gs))
    a_qdq = y.view(np.float16).astype(np.float64) if fp16 else bf16_bits_to_f64(y)
    w = dequant_nvfp4(w_codes, w_scales, w_global_scale)
    return a_exact @ w.T, a_qdq @ w.T, np.abs(a_exact) @ np.abs(w).T


def random_nvfp4_weight(n: int, k: int, seed: int):
    """Uniform random E2M1 nibbles; E4M3 scales uniform over the normal range
    [2^-6, 448] in log space (as a quantiser emits for a layer's groups), and a
    weight tensor scale of 1/2048."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    exp = rng.integers(1, 16, size=(n, k // 16))
    man = rng.integers(0, 8, size=(n, k // 16))
    man = np.where(exp == 15, np.minimum(man, 6), man)          # 0x7F is NaN
    scales = ((exp << 3) | man).astype(np.uint8)
    return codes, scales, 1.0 / 2048
