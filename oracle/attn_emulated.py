"""CPU restatement of the reference's EMULATED Sage3 attention path.

TEST INFRASTRUCTURE ONLY (tests/).  Nothing in the package imports it.

oracle/attn.py states the numerics this build's kernels implement (real E2M1
codes for every FP4 operand).  This module states what the reference itself
computes for its emulated configs ("nvfp4", "mxfp4"), operation by operation
and with every intermediate rounded to the type the reference holds it in, so
that the distance between the two definitions can be measured on any input
and the reference's accumulator modes (SAGE3_ACC_DTYPE) are covered:

  sage3/api.py:293-387        pad the sequence to 128 first, then smoothing,
                              host fake-quantisation, the kernel, trim, cast
  sage3/transforms.py:47-95   qk_smoothing (K mean over the padded sequence,
                              per-128-row Q means, delta_s = q_means @ k_c^T),
                              every op in the input dtype
  sage3/quantize.py:21-141    quantize_qk (blocks along D) / quantize_v (blocks
                              along the sequence): scale = dtype(amax / 6),
                              clamp 1e-8, E4M3 or E8M0 rounding of the scale
                              (the E8M0 log2 is itself rounded to the input
                              dtype, quant_primitives.py:140-151), clamp again,
                              dtype(x / scale), the 9-level grid, times scale
                              (fp32 result)
  sage3/quant_primitives.py:52-71  the 9 magnitudes {0, .5, .75, 1, 1.5, 2, 3,
                              4, 6}, ties upward (strict < thresholds)
  sage3/attention_kernel.py:15-195 the tiled online softmax with natural exp,
                              delta_s added before sm_scale, P quantised per
                              128-key tile, l = sum of the quantised P, and the
                              PV accumulator, its rescale and the final division
                              in the PV dtype of the accumulator mode
                              (ACC_DTYPE_MAP, api.py:25-35)
  sage3/p_quant_kernels.py:37-150  p_quant_nvfp4 (p * 2688, E4M3 scale per 16,
                              2688 left in) and p_quant_mxfp4 (E8M0 scale per
                              32, divided by 2688 at the end)

Roundings are modelled as the reference's CPU torch ops make them: an op on
bf16/fp16 operands is computed in fp32 and rounded to nearest even.  Dots and
reductions accumulate in float64 and round once, where the reference
accumulates in fp32 (on the GPU with TF32 operands, exact for these
fake-quantised values), so an output can differ in its last bit.

Pinned by tests/test_oracle_attn_golden.py against tests/golden/attn_reference.npz,
which holds outputs of the unmodified reference (tests/golden/make_attn_golden.py).
"""

from __future__ import annotations

import numpy as np

# ACC_DTYPE_MAP (sage3/api.py:25-35): mode -> dtype of the PV dot operands,
# the output accumulator and the final division; the QK dot and the softmax
# state stay fp32 in the modes covered here.
PV_DTYPE = {"fp32": "f32", "bf16_pv_only": "bf16", "fp16_pv_only": "f16"}

# per emulated config: (block size, scale rounding), the same for Q/K, V and P
# (sage3/quant_config.py:161-197)
EMULATED = {"nvfp4": (16, "e4m3"), "mxfp4": (32, "e8m0")}

COMBINED_MAX = 2688.0  # 448 * 6 (p_quant_kernels.py:60-62)
_GRID_EDGES = np.array([0.25, 0.625, 0.875, 1.25, 1.75, 2.5, 3.5, 5.0])
_GRID_VALUES = np.array([0.0, 0.5, 0.75, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64).astype(np.float32)


def _bf16(x) -> np.ndarray:
    """Round to bfloat16 (through fp32, as torch's CPU bf16 ops do), nearest even."""
    b = _f32(x).view(np.uint32).astype(np.uint64)
    r = (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    out = r.view(np.float32)
    return np.where(np.isnan(out), np.float32(np.nan), out)


def _f16(x) -> np.ndarray:
    return _f32(x).astype(np.float16).astype(np.float32)


def rnd(x, dt: str) -> np.ndarray:
    """x rounded to dtype dt ("bf16", "f16" or "f32"), returned as float32."""
    return {"bf16": _bf16, "f16": _f16, "f32": _f32}[dt](x)


def _e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn -> fp32, nearest even; beyond 448 gives NaN, as
    torch's cast does (quant_primitives.py:115-121)."""
    x = np.asarray(x, np.float64)
    a = np.abs(x)
    _, ex = np.frexp(np.maximum(a, 2.0 ** -6))
    step = np.where(a < 2.0 ** -6, 2.0 ** -9, np.exp2(ex - 4.0))
    q = np.round(a / step) * step  # half to even
    q = np.where(q > 448.0, np.nan, q)
    return np.copysign(q, x).astype(np.float32)


def grid9(x: np.ndarray) -> np.ndarray:
    """apply_e2m1_quantization (quant_primitives.py:52-71): nearest of the 9
    magnitudes, a value on a midpoint goes up, sign kept (fp32)."""
    x = np.asarray(x, np.float32)
    idx = np.searchsorted(_GRID_EDGES, np.abs(x), side="right")
    return (np.where(x >= 0, 1.0, -1.0) * _GRID_VALUES[idx]).astype(np.float32)


def _round_scale(sc: np.ndarray, how: str, dt: str) -> np.ndarray:
    """round_to_e4m3_torch / round_to_e8m0_torch on a dtype-dt scale tensor."""
    if how == "e4m3":
        return rnd(_e4m3(sc), dt)
    l2 = rnd(np.log2(np.maximum(np.abs(sc), np.float32(2.0 ** -127))), dt)
    return rnd(np.exp2(np.clip(np.ceil(l2), -127, 127)), dt)


def fake_quant(x: np.ndarray, block: int, how: str, dt: str) -> np.ndarray:
    """quantize_qk on x [..., K] with blocks along the last axis (quantize_v is
    this on the transposed V), x holding dtype-dt values; fp32 result."""
    sh = x.shape
    assert sh[-1] % block == 0
    xb = x.reshape(*sh[:-1], sh[-1] // block, block)
    eps = rnd(1e-8, dt)
    sc = rnd(np.abs(xb).max(axis=-1) / np.float32(6.0), dt)
    sc = np.maximum(sc, eps)
    sc = np.maximum(_round_scale(sc, how, dt), eps)
    with np.errstate(divide="ignore", invalid="ignore"):  # fp16 rounds the 1e-8 floor to 0
        xn = rnd(xb / sc[..., None], dt)
    return _f32(grid9(xn) * sc[..., None]).reshape(sh)


def prepass(q: np.ndarray, k: np.ndarray, v: np.ndarray, config: str, dt: str):
    """One (batch, head): q, k, v float32 [L, D] holding dtype-dt values.
    Returns the fake-quantised Q, K, V [Lp, D] (fp32), delta_s [G, Lp] (fp32)
    and Lp, for api.py:293-343 with qk_smoothing."""
    block, how = EMULATED[config]
    L, D = q.shape
    Lp = (L + 127) // 128 * 128
    pad = lambda a: np.concatenate([a, np.zeros((Lp - L, D), np.float32)])  # noqa: E731
    q, k, v = pad(q), pad(k), pad(v)
    # transforms.py:63-93 on the padded sequence
    kc = rnd(k - rnd(k.astype(np.float64).mean(axis=0), dt), dt)
    G = Lp // 128
    qmeans = rnd(q.reshape(G, 128, D).astype(np.float64).mean(axis=1), dt)
    qs = rnd(q - np.repeat(qmeans, 128, axis=0), dt)
    ds = rnd(qmeans.astype(np.float64) @ kc.astype(np.float64).T, dt)
    qd = fake_quant(qs, block, how, dt)
    kd = fake_quant(kc, block, how, dt)
    vd = np.ascontiguousarray(fake_quant(np.ascontiguousarray(v.T), block, how, dt).T)
    return qd, kd, vd, ds, Lp


def p_quant(p: np.ndarray, config: str) -> np.ndarray:
    """p_quant_nvfp4 / p_quant_mxfp4 on a [rows, 128] fp32 tile."""
    block, how = EMULATED[config]
    rows, w = p.shape
    p1 = _f32(p * np.float32(COMBINED_MAX)).reshape(rows, w // block, block)
    b = _f32(np.maximum(_f32(p1.max(axis=-1) / np.float32(6.0)), np.float32(1e-8)))
    if how == "e4m3":
        s = _e4m3(b)
    else:
        s = _f32(np.exp2(np.clip(np.ceil(_f32(np.log2(b))), -127, 127)))
    with np.errstate(divide="ignore", invalid="ignore"):  # a zero E4M3 scale gives 0 codes, as in the reference
        pq = _f32(grid9(_f32(p1 / s[..., None])) * s[..., None])
    if how == "e8m0":
        pq = _f32(pq / np.float32(COMBINED_MAX))
    return pq.reshape(rows, w)


def flash(qd, kd, vd, ds, sm_scale: float, config: str, acc: str) -> np.ndarray:
    """tiled_online_attention_kernel (attention_kernel.py:15-195), non-causal,
    128 x 128 tiles over the padded length; returns O [Lp, D] as the fp32
    values the kernel stores (already rounded to the PV dtype)."""
    pv = PV_DTYPE[acc]
    Lp, D = qd.shape
    G = Lp // 128
    group = np.minimum(np.arange(Lp) // 128, G - 1) if G > 1 else np.zeros(Lp, np.int64)
    scale = np.float32(sm_scale)
    m = np.full(Lp, -np.inf, np.float32)
    l = np.zeros(Lp, np.float32)
    o = np.zeros((Lp, D), np.float32)
    vp = rnd(vd, pv)
    for n0 in range(0, Lp, 128):
        s = _f32(qd.astype(np.float64) @ kd[n0:n0 + 128].astype(np.float64).T)
        s = _f32(s + ds[group, n0:n0 + 128])
        s = _f32(s * scale)
        m_new = np.maximum(m, s.max(axis=1))
        with np.errstate(invalid="ignore"):
            alpha = _f32(np.exp(_f32(m - m_new)))
        alpha = np.where(np.isneginf(m), np.float32(0.0), alpha)
        o = rnd(o * rnd(alpha, pv)[:, None], pv)
        p = _f32(np.exp(_f32(s - m_new[:, None])))
        pq = p_quant(p, config)
        pvt = rnd(_f32(rnd(pq, pv).astype(np.float64) @ vp[n0:n0 + 128].astype(np.float64)), pv)
        l = _f32(_f32(l * alpha) + _f32(pq.astype(np.float64).sum(axis=1)))
        m = m_new
        o = rnd(o + pvt, pv)
    # with fp16_pv_only, l (which carries the factor 2688 of p_quant_nvfp4)
    # can pass 65504 and round to inf in fp16: the reference then stores a
    # zero row, and so does this restatement
    with np.errstate(over="ignore"):
        return rnd(o / rnd(l, pv)[:, None], pv)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, sm_scale: float, config: str = "nvfp4",
              acc: str = "bf16_pv_only", f16: bool = False) -> np.ndarray:
    """The reference's sageattn3_standalone(q, k, v, config=config, acc_dtype=acc)
    for one (batch, head), non-causal: q, k, v float32 [L, D] holding bf16
    (fp16 if f16) values; returns O [L, D] rounded to the input dtype."""
    dt = "f16" if f16 else "bf16"
    qd, kd, vd, ds, _ = prepass(q, k, v, config, dt)
    return rnd(flash(qd, kd, vd, ds, sm_scale, config, acc)[: q.shape[0]], dt)
