"""CPU restatement of the reference's EMULATED Sage3 attention path.

TEST INFRASTRUCTURE ONLY (tests/).  Nothing in the package imports it.

oracle/attn.py states the numerics this build's kernels implement (the
reference's own grid for the emulated E8M0 configs, real E2M1 codes for
nvfp4 and mxfp4_s1_e4m3).  This module states what the reference itself
computes for its emulated configs (every config of sage3/quant_config.py:161-311
that runs the generic Triton kernel), operation by operation
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
  sage3/p_quant_kernels.py:37-283  p_quant_nvfp4 (p * 2688, E4M3 scale per 16,
                              2688 left in), p_quant_mxfp4 (E8M0 scale per
                              32, divided by 2688 at the end), and the
                              single-level mxfp4_s1, mxfp4_s1_e4m3 (E4M3 scale
                              floored at 2^-9) and mxfp8_s1 (E4M3 data)
  sage3/transforms.py:120-138 v_smoothing (V centred on its mean over the
                              padded sequence, the mean added to the output)

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

# QuantConfigs of the emulated configs (sage3/quant_config.py:161-266):
# name -> (block size along the quantised axis, scale rounding, data format, fp_max)
QUANT = {
    "nvfp4": (16, "e4m3", "e2m1", 6.0),
    "mxfp4": (32, "e8m0", "e2m1", 6.0),
    "mxfp4_s1": (32, "e8m0", "e2m1", 6.0),
    "mxfp8_s1": (32, "e8m0", "e4m3", 448.0),
    "mxfp4_s1_e4m3": (32, "e4m3", "e2m1", 6.0),
}

# AttentionConfigs (quant_config.py:174-311): config -> (Q/K QuantConfig,
# V QuantConfig, P-quant function of p_quant_kernels.py, V smoothing)
CONFIGS = {
    "nvfp4": ("nvfp4", "nvfp4", "nvfp4", False),
    "mxfp4": ("mxfp4", "mxfp4", "mxfp4", False),
    "mxfp4_s1": ("mxfp4_s1", "mxfp4_s1", "mxfp4_s1", False),
    "mxfp8_s1": ("mxfp8_s1", "mxfp8_s1", "mxfp8_s1", False),
    "mxfp4_s1_2level": ("mxfp4_s1", "mxfp4_s1", "mxfp4", False),
    "mxfp4_s1_e4m3": ("mxfp4_s1_e4m3", "mxfp4_s1_e4m3", "mxfp4_s1_e4m3", False),
    "mixed_fp8qk_fp4pv": ("mxfp8_s1", "mxfp4_s1", "mxfp4_s1", False),
    "mixed_fp4qk_fp8pv": ("mxfp4_s1", "mxfp8_s1", "mxfp8_s1", False),
    "mxfp4_s1_vsmooth": ("mxfp4_s1", "mxfp4_s1", "mxfp4_s1", True),
    "mixed_fp8qk_fp4pv_vs": ("mxfp8_s1", "mxfp4_s1", "mxfp4_s1", True),
    "mixed_fp4qk_fp8pv_vs": ("mxfp4_s1", "mxfp8_s1", "mxfp8_s1", True),
}

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


def fake_quant(x: np.ndarray, quant: str, dt: str) -> tuple[np.ndarray, str]:
    """quantize_qk with QuantConfig `quant` on x [..., K], blocks along the last
    axis (quantize_v is this on the transposed V), x holding dtype-dt values.
    Returns the values and the dtype the reference holds them in: fp32 for
    E2M1 data (the grid's sign tensor is fp32), the input dtype for E4M3 data
    (apply_e4m3_quantization_torch casts back to it; the products are exact)."""
    block, how, data, fp_max = QUANT[quant]
    sh = x.shape
    assert sh[-1] % block == 0
    xb = x.reshape(*sh[:-1], sh[-1] // block, block)
    eps = rnd(1e-8, dt)
    sc = rnd(np.abs(xb).max(axis=-1) / np.float32(fp_max), dt)
    sc = np.maximum(sc, eps)
    sc = np.maximum(_round_scale(sc, how, dt), eps)
    with np.errstate(divide="ignore", invalid="ignore"):  # fp16 rounds the 1e-8 floor to 0
        xn = rnd(xb / sc[..., None], dt)
    if data == "e4m3":
        return rnd(rnd(_e4m3(xn), dt) * sc[..., None], dt).reshape(sh), dt
    return _f32(grid9(xn) * sc[..., None]).reshape(sh), "f32"


def prepass(q: np.ndarray, k: np.ndarray, v: np.ndarray, config: str, dt: str):
    """One (batch, head): q, k, v float32 [L, D] holding dtype-dt values.
    Returns the fake-quantised Q, K, V [Lp, D] (fp32 values), delta_s [G, Lp]
    (fp32), the dtype the reference holds the quantised Q in (its output
    buffer has that dtype) and V's mean ([D], None without V smoothing), for
    api.py:293-343 with the config's pre-transforms."""
    qk_quant, pv_quant, _, vsmooth = CONFIGS[config]
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
    vmean = None
    if vsmooth:  # transforms.py:120-138, also over the padded sequence
        vmean = rnd(v.astype(np.float64).mean(axis=0), dt)
        v = rnd(v - vmean, dt)
    qd, out_dt = fake_quant(qs, qk_quant, dt)
    kd, _ = fake_quant(kc, qk_quant, dt)
    vd = np.ascontiguousarray(fake_quant(np.ascontiguousarray(v.T), pv_quant, dt)[0].T)
    return qd, kd, vd, ds, out_dt, vmean


def _e8m0_f32(b: np.ndarray) -> np.ndarray:
    """round_to_e8m0_triton on a positive fp32 value (quant_primitives.py:123-137)."""
    return _f32(np.exp2(np.clip(np.ceil(_f32(np.log2(b))), -127, 127)))


def p_quant(p: np.ndarray, kind: str) -> np.ndarray:
    """The P-quant function `kind` of p_quant_kernels.py on a [rows, 128] fp32
    tile: the two-level nvfp4 / mxfp4 (p * 2688 first) or the single-level
    mxfp4_s1 / mxfp4_s1_e4m3 / mxfp8_s1."""
    rows, w = p.shape
    block = 16 if kind == "nvfp4" else 32
    two_level = kind in ("nvfp4", "mxfp4")
    p1 = _f32(p * np.float32(COMBINED_MAX)) if two_level else _f32(p)
    p1 = p1.reshape(rows, w // block, block)
    fp_max = np.float32(448.0 if kind == "mxfp8_s1" else 6.0)
    b = _f32(np.maximum(_f32(p1.max(axis=-1) / fp_max), np.float32(1e-8)))
    if kind == "nvfp4":
        s = _e4m3(b)
    elif kind == "mxfp4_s1_e4m3":
        s = np.maximum(_e4m3(b), np.float32(2.0 ** -9))
    else:
        s = _e8m0_f32(b)
    with np.errstate(divide="ignore", invalid="ignore"):  # a zero E4M3 scale gives 0 codes, as in the reference
        pm = _f32(p1 / s[..., None])
    codes = _e4m3(pm) if kind == "mxfp8_s1" else grid9(pm)
    pq = _f32(codes * s[..., None])
    if kind == "mxfp4":
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
        pq = p_quant(p, CONFIGS[config][2])
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
    (fp16 if f16) values; returns O [L, D] rounded to the input dtype.
    The kernel stores O / l into a buffer of the quantised Q's dtype
    (attention_kernel.py:259, tl.store's cast), V's mean is added in that
    dtype (api.py:369-374), and the result is cast to the input dtype."""
    dt = "f16" if f16 else "bf16"
    qd, kd, vd, ds, out_dt, vmean = prepass(q, k, v, config, dt)
    o = rnd(flash(qd, kd, vd, ds, sm_scale, config, acc), out_dt)
    if vmean is not None:
        o = rnd(o + vmean, out_dt)
    return rnd(o[: q.shape[0]], dt)
