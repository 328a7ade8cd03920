"""CPU oracle of the Sage3 FP4 / FP8 attention (the reference's mxfp4_hw and mxfp8_hw paths).

TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py baselines).

Restates, in numpy (float64 accumulation):
  - qk_smoothing (src/vllm_qdq_plugin/sage3_attn/sage3/transforms.py:47-95)
    applied before padding, as the mxfp4_hw branch does (sage3/api.py:161-182),
    with every bf16 op rounded to bf16;
  - quantize_to_mxfp4 of q_s, k_c (along D) and V (along the sequence)
    (sage3/mxfp4_hw_kernel.py:73-116) via the C oracle, pinned to the
    reference's own outputs by tests/golden/mxfp4_hw_quant.npz;
  - the flash loop of _mxfp4_attn_fwd_inner (mxfp4_hw_kernel.py:205-282):
    S = deq(Q) deq(K)^T + delta_s, base-2 online softmax with
    qk_scale = sm_scale * log2(e), l += sum of the unquantised p, P quantised
    per 32 keys with E8M0 scale 2^ceil(log2(max p / 6)) and round-to-nearest-even
    E2M1, O += deq(P) deq(V), O / l.
The quantised P depends on the running max at each key tile, so the tile
width is a parameter: the sm_100a kernel uses 128, the reference kernel 64.
Keys beyond L are masked (mask_padding=True) or, as in the reference,
attended as zero keys (mask_padding=False).
The reference's emulated E8M0 configs (mxfp4, mxfp4_s1, mxfp8_s1, the mixed
and V-smoothed ones) use its own quantize_qk / quantize_v steps (formats "g9",
"e8", from oracle/attn_emulated.py) and, for "g9" P, its 9-level grid with ties
upward; this is what the sm_100a kernels compute for them.
The mxfp8_hw path (sage3/api.py:114-160, mxfp8_hw_kernel.py:37-246) is the
same with quantize_to_mxfp8 (via the C oracle, pinned by
tests/golden/mxfp8_hw_quant.npz) and P quantised to E4M3 with
E8M0 2^ceil(log2(max p / 448)) per 32 keys (round-to-nearest-even).
"""

from __future__ import annotations

import numpy as np

from . import attn_emulated as _ae
from . import qdq as oq

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float64)
LOG2E = 1.4426950408889634


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float values to bf16 (nearest even), returned as float32.  This
    is the rounding of torch's bf16 cast, which the reference's torch code
    applies after every bf16 operation; the cast is used here for speed."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round to fp16 (nearest even; numpy's conversion from float64 rounds
    once), returned as float32: the reference's torch ops on fp16 inputs."""
    return np.asarray(x, np.float64).astype(np.float16).astype(np.float32)


def round16(x: np.ndarray, f16: bool = False) -> np.ndarray:
    """Round to the 16-bit input dtype: fp16 if f16, else bf16."""
    return f16_round(x) if f16 else bf16_round(x)


def bits_to_f32(bits: np.ndarray, f16: bool = False) -> np.ndarray:
    """uint16 bit patterns of fp16 (f16) or bf16 values -> float32."""
    if f16:
        return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)
    return bf16_bits_to_f32(bits)


def _e4m3_table() -> np.ndarray:
    b = np.arange(256)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    mag = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8) * np.exp2(e - 7.0))
    mag[(b & 0x7F) == 0x7F] = np.nan
    return np.where(b & 0x80, -mag, mag)


E4M3 = _e4m3_table()


def _deq8(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """E4M3 bytes [..., K] with E8M0 scales per 32 -> float64."""
    return E4M3[codes] * np.repeat(np.exp2(scales.astype(np.float64) - 127.0), 32, axis=-1)


def _deq(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    lo = E2M1[codes & 0xF]
    hi = E2M1[codes >> 4]
    vals = np.stack([lo, hi], axis=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)
    sc = np.exp2(scales.astype(np.float64) - 127.0)
    return vals * np.repeat(sc, 32, axis=-1)


def _rne_e2m1(v: np.ndarray) -> np.ndarray:
    a = np.minimum(np.abs(v), 6.0)
    q = np.where(a <= 0.25, 0.0, np.where(a < 0.75, 0.5, np.where(a <= 1.25, 1.0,
        np.where(a < 1.75, 1.5, np.where(a <= 2.5, 2.0, np.where(a < 3.5, 3.0,
        np.where(a <= 5.0, 4.0, 6.0)))))))
    return np.copysign(q, v)


def _rna_e2m1(v: np.ndarray) -> np.ndarray:
    """Round-half-away onto the E2M1 grid (the reference's _float_to_e2m1_nibble
    thresholds, mxfp4_hw_kernel.py:43-61), clamped to 6."""
    a = np.minimum(np.abs(v), 6.0)
    q = np.where(a < 0.25, 0.0, np.where(a < 0.75, 0.5, np.where(a < 1.25, 1.0,
        np.where(a < 1.75, 1.5, np.where(a < 2.5, 2.0, np.where(a < 3.5, 3.0,
        np.where(a < 5.0, 4.0, 6.0)))))))
    return np.copysign(q, v)


def e4m3_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn -> fp32 for 0 <= x <= 448, round-to-nearest-even."""
    x = np.minimum(np.asarray(x, np.float64), 448.0)
    _, ex = np.frexp(np.maximum(x, 2.0 ** -6))  # x = m * 2^ex, m in [0.5, 1)
    step = np.where(x < 2.0 ** -6, 2.0 ** -9, np.exp2(ex - 1 - 3.0))
    return (np.round(x / step) * step).astype(np.float32)  # np.round: half to even


def nv_quant_deq(x: np.ndarray, block: int = 16, f16: bool = False) -> np.ndarray:
    """NVFP4 of the reference's nvfp4 QuantConfig (quantize.py:21-81 with
    round_to_e4m3) on the hardware grid, per 16 along the last axis:
    scale = e4m3(max(bf16(amax / 6), 1e-8)), codes of the exact quotient
    x / scale rounded half away from zero (the reference's own steps use a
    bf16 quotient and a 9-level grid no FP4 hardware has; parity with them is
    by tolerance), dequantised; a zero scale zeroes the block.  block=32 gives
    the mxfp4_s1_e4m3 QuantConfig (quant_config.py:246-255), the same steps per
    32.  With fp16 inputs (f16) the scale is rounded to fp16 instead of bf16."""
    sh = x.shape
    xb = np.asarray(x, np.float32).reshape(*sh[:-1], sh[-1] // block, block)
    amax = np.abs(xb).max(axis=-1)
    sc = np.maximum(round16(amax / np.float32(6.0), f16), np.float32(1e-8))
    s = e4m3_round(sc).astype(np.float64)
    quot = xb.astype(np.float64) / np.where(s > 0, s, 1.0)[..., None]  # correctly rounded: exact at midpoints
    q = np.where(s[..., None] > 0, _rna_e2m1(quot), 0.0)
    return (q * s[..., None]).reshape(sh)


def _ceil_log2(r: np.ndarray) -> np.ndarray:
    m, e = np.frexp(r)  # r = m * 2^e, m in [0.5, 1)
    out = np.where(m == 0.5, e - 1, e).astype(np.int64)
    return np.where(r == 0, -127, out)


def _quant_deq(x: np.ndarray, fmt: str, f16: bool = False) -> np.ndarray:
    """Dequantised x [rows, K] in operand format fmt, blocks along K:
    "mx4" quantize_to_mxfp4, "nv4" NVFP4 per 16, "mx8" quantize_to_mxfp8,
    "nv4b32" E2M1 with an E4M3 scale per 32; "g9" / "e8" the reference's own
    emulated quantize_qk steps for its mxfp4 / mxfp8_s1 QuantConfigs (9-level
    grid or E4M3 codes, E8M0 per 32, scale arithmetic in the input dtype),
    restated in oracle/attn_emulated.py.  An all-zero fp16 group, whose
    reference scale underflows to 0, dequantises to 0 here, as the sm_100a
    pre-pass writes it."""
    if fmt in ("g9", "e8"):
        v, _ = _ae.fake_quant(np.asarray(x, np.float32), "mxfp4_s1" if fmt == "g9" else "mxfp8_s1",
                              "f16" if f16 else "bf16")
        return np.nan_to_num(v.astype(np.float64), nan=0.0)
    if fmt == "nv4":
        return nv_quant_deq(x, 16, f16)
    if fmt == "nv4b32":
        return nv_quant_deq(x, 32, f16)
    if fmt == "mx8":
        return _deq8(*oq.mxfp8_hw_quant(x))
    return _deq(*oq.mxfp4_hw_quant(x))


def prepass(q: np.ndarray, k: np.ndarray, v: np.ndarray, smoothing: bool = True, nv: bool = False,
            fp8: bool = False, qk_fmt: str | None = None, pv_fmt: str | None = None, vsmooth: bool = False,
            f16: bool = False):
    """q, k, v: float32 [L, D] holding bf16 values for one (batch, head).
    Returns (qd, kd, vd, ds): dequantised Q [Lp, D], K [Lp, D], V [Lp, D]
    (V quantised along the sequence) and delta_s [G, Lp] (zeros without
    smoothing).  nv selects NVFP4 blocks of 16 (E4M3) instead of MXFP4; fp8
    selects MXFP8 (quantize_to_mxfp8); qk_fmt / pv_fmt ("mx4", "nv4", "mx8")
    set the two operand formats separately.  vsmooth (transforms.py
    v_smoothing) quantises bf16(v - bf16(mean_L(v))); the mean is then the
    caller's to add to the output (see vmean()).  f16: the inputs are fp16
    values and every rounding of the smoothing is to fp16."""
    default = "nv4" if nv else ("mx8" if fp8 else "mx4")
    qk_fmt = qk_fmt or default
    pv_fmt = pv_fmt or default
    L, D = q.shape
    Lp = (L + 127) // 128 * 128
    G = Lp // 128
    if smoothing:
        kmean = round16(k.astype(np.float64).mean(axis=0), f16)
        kc = round16(k - kmean, f16)
        qpad = np.zeros((Lp, D), np.float32)
        qpad[:L] = q
        qmeans = round16(qpad.reshape(G, 128, D).astype(np.float64).mean(axis=1), f16)
        qs = round16(q - np.repeat(qmeans, 128, axis=0)[:L], f16)
        ds = round16(qmeans.astype(np.float64) @ kc.astype(np.float64).T, f16)  # [G, L]
    else:
        kc, qs = k, q
        ds = np.zeros((G, L), np.float32)
    pad = lambda a: np.concatenate([a, np.zeros((Lp - L, D), np.float32)])  # noqa: E731
    dsp = np.zeros((G, Lp), np.float64)
    dsp[:, :L] = ds
    if vsmooth:
        v = round16(v - vmean(v, f16), f16)
    return (_quant_deq(pad(qs), qk_fmt, f16), _quant_deq(pad(kc), qk_fmt, f16),
            _quant_deq(np.ascontiguousarray(pad(v).T), pv_fmt, f16).T, dsp)


def vmean(v: np.ndarray, f16: bool = False) -> np.ndarray:
    """dtype(mean over the sequence of v) [D] (transforms.py v_smoothing)."""
    return round16(v.astype(np.float64).mean(axis=0), f16)


def flash(qd, kd, vd, ds, L: int, sm_scale: float, block_n: int = 128, causal: bool = False,
          mask_padding: bool = True, nv: bool = False, emulated: bool = False,
          q_rows: slice | None = None, fp8: bool = False, pre: float | None = None,
          e4s32: bool = False, g9: bool = False) -> np.ndarray:
    """The attention loop on dequantised operands; returns O [L, D] float64
    (or the rows q_rows of it, for timing a slice of the query tiles).

    P handling: mxfp4_hw (nv=False, emulated=False): E8M0 per 32 of p, l = sum
    of unquantised p.  Emulated configs (emulated=True): p scaled by 448*6
    first, l = sum of the dequantised P (p_quant_kernels.py:37-150,
    attention_kernel.py:176-186); nv=True uses E4M3 per 16.  fp8=True: the
    mxfp8_hw kernel's P, E4M3 codes of min(p / 2^e, 448) with
    e = clamp(ceil(log2(max p / 448)), -127, 127) per 32, l = sum of p; with
    emulated=True the single-level emulated MXFP8 P (p_quant_mxfp8_s1): the
    same codes, l = sum of the dequantised P.  pre: the emulated prescale
    (448*6 by default, 1 for the single-level _s1 configs).  The emulated E8M0
    scales take the reference's max(., 1e-8) before the ceiling.  e4s32=True:
    p_quant_mxfp4_s1_e4m3 (p_quant_kernels.py:197-232), E2M1 with the scale
    max(e4m3(max(b / 6, 1e-8)), 2^-9) per 32.  g9=True (with emulated): the
    reference's p_quant_mxfp4 / p_quant_mxfp4_s1 exactly, codes on its 9-level
    grid with ties upward instead of round-to-nearest-even E2M1."""
    Lp, D = kd.shape
    n_keys = L if mask_padding else Lp
    qk_scale = sm_scale * LOG2E
    rows = np.arange(Lp)[q_rows] if q_rows is not None else np.arange(Lp)
    qd = qd[rows]
    nq = len(rows)
    m = np.full(nq, -np.inf)
    l = np.zeros(nq)
    acc = np.zeros((nq, D))
    group = rows // 128
    if pre is None or not emulated:
        pre = 2688.0 if emulated else 1.0
    for n0 in range(0, n_keys, block_n):
        n1 = min(n0 + block_n, Lp)
        s = qd @ kd[n0:n1].T + ds[group, n0:n1]
        keys = np.arange(n0, n1)
        valid = np.broadcast_to(keys[None, :] < n_keys, s.shape)
        if causal:
            valid = valid & (keys[None, :] <= rows[:, None])
        s = np.where(valid, s, -np.inf)
        m_new = np.maximum(m, s.max(axis=1) * qk_scale)
        alpha = np.where(np.isneginf(m), 0.0, np.exp2(m - m_new))
        p = np.where(valid, np.exp2(s * qk_scale - m_new[:, None]), 0.0)
        acc = acc * alpha[:, None]
        w = n1 - n0
        p1 = p * pre
        if fp8:
            pg = p1.reshape(nq, w // 32, 32)
            e = np.clip(_ceil_log2(pg.max(axis=2) / 448.0), -127, 127)
            if emulated:
                e = np.maximum(e, -26)  # ceil(log2(1e-8))
            sc = np.exp2(e.astype(np.float64))[:, :, None]
            pq = (e4m3_round(pg / sc).astype(np.float64) * sc).reshape(nq, w)
        elif e4s32:
            pg = p1.reshape(nq, w // 32, 32)
            sc = np.maximum(e4m3_round(np.maximum(pg.max(axis=2) / 6.0, 1e-8)), 2.0 ** -9)
            sc = sc.astype(np.float64)[:, :, None]
            pq = (_rne_e2m1(pg * (1.0 / sc)) * sc).reshape(nq, w)
        elif nv:
            pg = p1.reshape(nq, w // 16, 16)
            sc = e4m3_round(np.maximum(pg.max(axis=2) / 6.0, 1e-8)).astype(np.float64)[:, :, None]
            inv = np.where(sc > 0, 1.0 / np.where(sc > 0, sc, 1), 0.0)
            pq = (_rne_e2m1(pg * inv) * sc).reshape(nq, w)
        else:
            pg = p1.reshape(nq, w // 32, 32)
            e = np.clip(_ceil_log2(pg.max(axis=2) / 6.0), -127, 127)
            if emulated:
                e = np.maximum(e, -26)  # ceil(log2(1e-8))
            sc = np.exp2(e.astype(np.float64))[:, :, None]
            codes = _ae.grid9(pg / sc).astype(np.float64) if g9 else _rne_e2m1(pg / sc)
            pq = (codes * sc).reshape(nq, w)
        l = l * alpha + (pq.sum(axis=1) if emulated else p.sum(axis=1))
        acc = acc + pq @ vd[n0:n1]
        m = m_new
    return (acc / l[:, None])[rows < L]


# config -> (Q/K format, P/V format, emulated P, prescale, V smoothing, QK smoothing)
# (reference: sage3/quant_config.py:161-330 and the hardware branches of sage3/api.py)
CONFIGS = {
    "mxfp4_hw": ("mx4", "mx4", False, 1.0, False, True),
    "mxfp4": ("g9", "g9", True, 2688.0, False, True),
    "mxfp4_s1_2level": ("g9", "g9", True, 2688.0, False, True),
    "nvfp4": ("nv4", "nv4", True, 2688.0, False, True),
    "mxfp8_hw": ("mx8", "mx8", False, 1.0, False, True),
    "mxfp4_s1": ("g9", "g9", True, 1.0, False, True),
    "mxfp8_s1": ("e8", "e8", True, 1.0, False, True),
    "mixed_fp8qk_fp4pv": ("e8", "g9", True, 1.0, False, True),
    "mixed_fp4qk_fp8pv": ("g9", "e8", True, 1.0, False, True),
    "mixed_mxfp8qk_mxfp4pv_hw": ("mx8", "mx4", False, 1.0, False, False),
    "mixed_mxfp4qk_mxfp8pv_hw": ("mx4", "mx8", False, 1.0, False, False),
    "mxfp4_s1_vsmooth": ("g9", "g9", True, 1.0, True, True),
    "mixed_fp8qk_fp4pv_vs": ("e8", "g9", True, 1.0, True, True),
    "mixed_fp4qk_fp8pv_vs": ("g9", "e8", True, 1.0, True, True),
    "mxfp4_s1_e4m3": ("nv4b32", "nv4b32", True, 1.0, False, True),
}

def p_flags(pv_fmt: str) -> dict:
    """flash()'s P-quantisation switches for a P/V operand format."""
    return {"nv": pv_fmt == "nv4", "fp8": pv_fmt in ("mx8", "e8"), "e4s32": pv_fmt == "nv4b32",
            "g9": pv_fmt == "g9"}


# Key tile of the reference's online softmax per config: the mxfp4_hw kernel
# launches with BLOCK_N = 64 (sage3/mxfp4_hw_kernel.py:437); the emulated
# configs' attention kernel requires tile_size_k = 128 (attention_kernel.py:249-253);
# the mxfp8_hw and mixed hardware kernels launch with BLOCK_N = 64
# (sage3/mxfp8_hw_kernel.py:341 and the mixed kernels' launchers).
REF_BLOCK_N = {name: (128 if cfg[2] else 64) for name, cfg in CONFIGS.items()}


def attention(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, sm_scale: float,
              block_n: int | None = None, causal: bool = False, smoothing: bool = True,
              mask_padding: bool = True, config: str = "mxfp4_hw", f16: bool = False) -> np.ndarray:
    """q/k/v: uint16 bf16 (fp16 if f16) bit patterns [L, H, D] (NHD with B = 1);
    returns O [L, H, D].  block_n defaults to the reference's key tile for the
    config (REF_BLOCK_N)."""
    qk_fmt, pv_fmt, emulated, pre, vsmooth, qk_smooth = CONFIGS[config]
    smoothing = smoothing and qk_smooth
    if block_n is None:
        block_n = REF_BLOCK_N[config]
    L, H, D = q_bits.shape
    out = np.zeros((L, H, D))
    for h in range(H):
        q = bits_to_f32(q_bits[:, h], f16)
        k = bits_to_f32(k_bits[:, h], f16)
        v = bits_to_f32(v_bits[:, h], f16)
        qd, kd, vd, ds = prepass(q, k, v, smoothing, qk_fmt=qk_fmt, pv_fmt=pv_fmt, vsmooth=vsmooth, f16=f16)
        out[:, h] = flash(qd, kd, vd, ds, L, sm_scale, block_n, causal, mask_padding, emulated=emulated, pre=pre,
                          **p_flags(pv_fmt))
        if vsmooth:
            out[:, h] += vmean(v, f16)
    return out


def attention_rows(q_bits: np.ndarray, k_bits: np.ndarray, v_bits: np.ndarray, sm_scale: float,
                   rows: np.ndarray, config: str = "mxfp4_hw", block_n: int | None = None,
                   mask_padding: bool = True, f16: bool = False) -> np.ndarray:
    """attention() of one head ([L, 1, D] bit patterns) for the query rows
    `rows` only: the pre-pass over the whole sequence, then the flash loop on
    each 128-row query tile that holds a requested row.  Returns O [len(rows), D]."""
    qk_fmt, pv_fmt, emulated, pre, vsmooth, qk_smooth = CONFIGS[config]
    if block_n is None:
        block_n = REF_BLOCK_N[config]
    L = q_bits.shape[0]
    q, k, v = (bits_to_f32(t[:, 0], f16) for t in (q_bits, k_bits, v_bits))
    qd, kd, vd, ds = prepass(q, k, v, qk_smooth, qk_fmt=qk_fmt, pv_fmt=pv_fmt, vsmooth=vsmooth, f16=f16)
    rows = np.asarray(rows)
    out = np.zeros((len(rows), q.shape[1]))
    for t in np.unique(rows // 128):
        o = flash(qd, kd, vd, ds, L, sm_scale, block_n, False, mask_padding, emulated=emulated,
                  q_rows=slice(128 * t, 128 * t + 128), pre=pre, **p_flags(pv_fmt))
        sel = rows // 128 == t
        out[sel] = o[rows[sel] - 128 * t]
        if vsmooth:
            out[sel] += vmean(v, f16)
    return out


def exact_attention(q_bits, k_bits, v_bits, sm_scale: float, causal: bool = False, f16: bool = False) -> np.ndarray:
    """Unquantised float64 softmax attention (the accuracy reference)."""
    L, H, D = q_bits.shape
    out = np.zeros((L, H, D))
    for h in range(H):
        q = bits_to_f32(q_bits[:, h], f16).astype(np.float64)
        k = bits_to_f32(k_bits[:, h], f16).astype(np.float64)
        v = bits_to_f32(v_bits[:, h], f16).astype(np.float64)
        s = q @ k.T * sm_scale
        if causal:
            s = np.where(np.arange(L)[None, :] <= np.arange(L)[:, None], s, -np.inf)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out[:, h] = (p / p.sum(axis=1, keepdims=True)) @ v
    return out


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))
