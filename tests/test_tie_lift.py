"""CPU: the E2M1 encoders' tie lift, exhaustively, for bf16 and fp16 inputs.

The pre-pass kernels (vllm-qdq-plugin_b200/csrc/attn_prepass.cu) encode with
the hardware's round-to-nearest-even cvt, while the reference rounds half away
from zero (sage3/mxfp4_hw_kernel.py:43-61 for E8M0-scaled groups, and this
build's exact-quotient rule for E4M3-scaled ones).  The kernels scale by
(1 + 2^-12) first, which lifts exact midpoints above and moves nothing else
across one.  Here that is checked for every 16-bit input value:
  E8M0:  every bf16 / fp16 x and every exponent e in [-40, 40]:
         RNE(f32(x * 2^-e * (1 + 2^-12))) == RHA(x * 2^-e)
  E4M3:  every bf16 / fp16 x and every positive E4M3 scale s:
         RNE(f32(x * f32(f32(1 / s) * (1 + 2^-12)))) == RHA(x / s)
with float32 arithmetic emulated by numpy (IEEE round-to-nearest-even) and
the cvt's satfinite (magnitudes above 6 give 6).  Codes are compared by
magnitude: a negative product that underflows to zero gives the code -0,
which dequantises like +0.
"""

from __future__ import annotations

import numpy as np
import pytest

GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
MID = (GRID[1:] + GRID[:-1]) / 2  # 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5


def _all_values(dtype: str) -> np.ndarray:
    bits = np.arange(1 << 16, dtype=np.uint32)
    if dtype == "fp16":
        vals = bits.astype(np.uint16).view(np.float16).astype(np.float64)
    else:
        vals = (bits << 16).view(np.float32).astype(np.float64)
    return vals[np.isfinite(vals)]


def _rha(a: np.ndarray) -> np.ndarray:
    """Magnitude code, round half away from zero (ties to the larger value)."""
    return np.minimum(np.searchsorted(MID, a, side="right"), 7)


def _rne(a: np.ndarray) -> np.ndarray:
    """Magnitude code, round to nearest, ties to the even code; satfinite."""
    lo = np.searchsorted(MID, a, side="left")     # a <= MID[lo]: code lo unless a is the tie MID[lo]
    code = np.minimum(lo, 7)
    tie = (lo < 7) & (a == MID[np.minimum(lo, 6)])
    even_up = (lo + 1) % 2 == 0                    # the tie's upper neighbour has the even code
    return np.where(tie & even_up, np.minimum(lo + 1, 7), code)


LIFT = np.float32(1.0 + 2.0 ** -12)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@np.errstate(over="ignore")  # huge x: the float32 product is inf, which the cvt saturates like the reference
def test_e8m0_lift_gives_round_half_away(dtype):
    x = np.abs(_all_values(dtype))
    for e in range(-40, 41):
        inv = np.float32(2.0 ** -e) * LIFT                      # exact: a power of two times LIFT
        y = (x * 2.0 ** -e)                                      # exact (float64)
        t = (x.astype(np.float32) * inv).astype(np.float32)      # the kernel's fma(x, inv, 0)
        assert np.array_equal(_rne(t.astype(np.float64)), _rha(y)), (dtype, e)


def _e4m3_positive() -> np.ndarray:
    out = []
    for b in range(1, 0x7F):      # 0x7F is NaN
        ex, man = b >> 3, b & 7
        out.append(man * 2.0 ** -9 if ex == 0 else (1 + man / 8) * 2.0 ** (ex - 7))
    return np.array(out)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@np.errstate(over="ignore")
def test_e4m3_lift_gives_round_half_away(dtype):
    x = np.abs(_all_values(dtype))
    x32 = x.astype(np.float32)
    for s in _e4m3_positive():
        inv = (np.float32(1.0) / np.float32(s)).astype(np.float32)
        inv = (inv * LIFT).astype(np.float32)
        t = (x32 * inv).astype(np.float32)
        want = _rha(x / s)            # float64 quotient: exact at midpoints, right side of them otherwise
        assert np.array_equal(_rne(t.astype(np.float64)), want), (dtype, s)


def test_helpers_round_as_defined():
    a = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 0.2, 0.3])
    assert _rha(a).tolist() == [1, 2, 3, 4, 5, 6, 7, 7, 0, 1]
    assert _rne(a).tolist() == [0, 2, 2, 4, 4, 6, 6, 7, 0, 1]
