"""CPU: the two arithmetic shortcuts the sm_100a kernels use to reproduce the
reference's emulated E8M0 quantisation, checked exhaustively against the
reference's own rules.

1. grid9_mag (csrc/attn_prepass.cu, csrc/attn_flash.cu): the reference's
   9-level grid {0, .5, .75, 1, 1.5, 2, 3, 4, 6} with ties upward
   (apply_e2m1_quantization, sage3/quant_primitives.py:52-71) as one fp32
   integer add and mask (round to one mantissa bit, ties up) above 0.5, two
   compares below, a cap at 6.  Restated here on the fp32 bit patterns and
   compared with the compare chain (oracle/attn_emulated.py:grid9) for every
   bf16 and fp16 value (the pre-pass applies it to values of the input dtype)
   and every fp32 value in [0.25, 8) (the P quantiser applies it to exp2
   results, at most 6 and a little).
2. emu8_quant32's scale exponent: the reference evaluates
   ceil(log2(sc)) on a bf16 / fp16 tensor, i.e. log2 rounded to fp32 and then
   to the tensor's dtype (quant_primitives.py:140-151); near a power of two that
   rounding can lower the ceiling by one.  The kernel takes log2 in double
   precision, rounds it once to fp32 and then to the dtype.  Checked equal to
   torch's own chain for every positive bf16 scale the reference can form
   (at least bf16(1e-8)) and every positive fp16 scale.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import attn_emulated as ae


def _grid9_mag_bits(a: np.ndarray) -> np.ndarray:
    """The kernels' grid9_mag on float32 a >= 0."""
    a = np.asarray(a, np.float32)
    r = ((a.view(np.uint32).astype(np.uint64) + 0x00200000) & 0xFFC00000).astype(np.uint32).view(np.float32)
    return np.where(a < 0.5, np.where(a < 0.25, 0.0, 0.5), np.minimum(r, 6.0)).astype(np.float32)


def _check_grid(a: np.ndarray) -> None:
    got = _grid9_mag_bits(a)
    want = ae.grid9(a)
    bad = got != want
    assert not bad.any(), (a[bad][:8], got[bad][:8], want[bad][:8])


def test_grid9_bit_rule_on_every_bf16_and_fp16_value():
    bf = (np.arange(0, 0x7F80, dtype=np.uint32) << 16).view(np.float32)  # every finite bf16 >= 0
    _check_grid(bf)
    hf = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)  # every finite fp16 >= 0
    _check_grid(hf)


def test_grid9_bit_rule_on_every_fp32_value_from_a_quarter_to_eight():
    lo = np.float32(0.25).view(np.uint32)
    hi = np.float32(8.0).view(np.uint32)
    step = 1 << 22
    for start in range(int(lo), int(hi), step):
        bits = np.arange(start, min(start + step, int(hi)), dtype=np.uint32)
        _check_grid(bits.view(np.float32))


def _kernel_exp(sc: np.ndarray, f16: bool) -> np.ndarray:
    """emu8_quant32's exponent: ceil(T(fp32(log2 in double))) for sc > 0."""
    lg = np.log2(sc.astype(np.float64)).astype(np.float32)
    t = torch.from_numpy(lg).to(torch.float16 if f16 else torch.bfloat16).float().numpy()
    return np.ceil(t)


def test_scale_exponent_rule_on_every_bf16_scale():
    sc = (np.arange(1, 0x7F80, dtype=np.uint32) << 16).view(np.float32)
    sc = sc[sc >= torch.tensor(1e-8).to(torch.bfloat16).item()]
    ref = torch.ceil(torch.log2(torch.from_numpy(sc).to(torch.bfloat16).clamp(min=2 ** -127))).float().numpy()
    assert np.array_equal(_kernel_exp(sc, False), ref)


def test_scale_exponent_rule_on_every_fp16_scale():
    sc = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    ref = torch.ceil(torch.log2(torch.from_numpy(sc).to(torch.float16))).float().numpy()
    assert np.array_equal(_kernel_exp(sc, True), ref)
