"""Golden outputs of the reference's own Sage3 attention, for the GPU parity
tests in tests/test_attn_reference_gpu.py and the CPU pin of oracle/attn.py in
tests/test_oracle_attn_golden.py.

Run inside the build container, where the reference checkout imports (CPU
only, a few minutes):

    python tests/golden/make_attn_golden.py --reference /path/to/vllm-qdq-plugin

It runs the reference's attention end to end on the CPU.  Its torch pre-pass
(qk_smoothing, quantize_qk / quantize_v, quantize_to_mxfp4 / _mxfp8, the
padding) runs as written, and its Triton kernels (sage3/attention_kernel.py,
sage3/mxfp4_hw_kernel.py, sage3/mxfp8_hw_kernel.py) run unmodified under
Triton's interpreter (TRITON_INTERPRET=1).  Triton 3.6's interpreter lacks
four things these kernels use; this script fills them in its own process,
without touching the reference:

  1. tl.dot_scaled: each operand is decoded (E2M1 nibbles, element 2j in the
     low nibble, or E4M3 bytes) and multiplied by 2^(E8M0 - 127) of its
     32-element group; the product of the decoded matrices is formed in
     float64 (every product of these operands is exact) and added to the fp32
     accumulator, as the tensor core does.  (The interpreter also hands the
     format strings to the semantic layer unwrapped; they are wrapped.)
  2. the inline-PTX `cvt.rn.satfinite.e2m1x2.f32` of mxfp4_hw_kernel.py:143-164:
     round to nearest even onto the E2M1 grid, saturating at 6; the first
     source operand goes to the high nibble, as the instruction packs it.
  3. bfloat16 arithmetic: the interpreter stores bf16 as raw 16-bit integers
     and would add, multiply, compare and multiply matrices on those integers;
     here every bf16 operation is done in fp32 and rounded to nearest even, and
     a bf16 matrix product accumulates in fp32, as the GPU does.
  4. downcasts: fp32 -> bf16 rounds to nearest even (the interpreter
     truncates) and fp32 -> fp8 e4m3 rounds to nearest even (the interpreter
     converts the integer value).
The mxfp8_hw module also asks Triton's active GPU driver for its torch device
when it is imported (mxfp8_hw_kernel.py:24); with no GPU a stand-in driver
answers "cpu".

Elementwise math (exp, exp2, log2, division) uses numpy's correctly rounded
fp32 functions where the GPU uses approximate ones; the fp32 dots are exact
where the GPU uses TF32, which for these fake-quantised operands (at most 8
significant bits) is exact too.  The outputs are therefore the reference's
results up to last-bit differences of fp32 math.

Fixture tests/golden/attn_reference.npz holds, per case: the reference output
(bf16 bits, as `sageattn3_standalone` returns it), the query rows it covers,
and a checksum of the seeded inputs, which the tests regenerate with
`case_inputs` below (torch's CPU generator is deterministic).
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name -> (config, acc_dtype, distribution, B, H, L, query tiles (None = all)[, head dim[, input dtype]])
CASES = {
    # config 4 (Wan-2.1): the reference's Blackwell kernel, 64-key steps
    "mxfp4_hw_L1024": ("mxfp4_hw", "fp32", "c4", 1, 2, 1024, None),
    "mxfp4_hw_L4608": ("mxfp4_hw", "fp32", "c4", 1, 1, 4608, None),
    # the full config-4 sequence: 75600 keys (the reference also attends its 48
    # zero padding keys), three query tiles including the ragged last one
    "mxfp4_hw_L75600": ("mxfp4_hw", "fp32", "c4", 1, 1, 75600, (0, 295, 590)),
    # config 5 (Flux): emulated NVFP4, bf16 PV accumulation
    "nvfp4_bf16pv_L1024": ("nvfp4", "bf16_pv_only", "c5", 1, 2, 1024, None),
    "nvfp4_bf16pv_L4608": ("nvfp4", "bf16_pv_only", "c5", 1, 1, 4608, None),
    # emulated MXFP4 (fp32 accumulation) and the hardware MXFP8 kernel
    "mxfp4_L1024": ("mxfp4", "fp32", "c4", 1, 2, 1024, None),
    "mxfp8_hw_L1024": ("mxfp8_hw", "fp32", "c4", 1, 2, 1024, None),
    # head dim 64, which the reference's hardware kernels take beside 128
    # (mxfp4_hw_kernel.py:439), and the emulated NVFP4 config at D = 64 (fp32
    # accumulation, which the reference allows below D = 128)
    "mxfp4_hw_D64_L1024": ("mxfp4_hw", "fp32", "c4", 1, 2, 1024, None, 64),
    "nvfp4_D64_L1024": ("nvfp4", "fp32", "c5", 1, 2, 1024, None, 64),
    # fp16 inputs: the reference's smoothing then runs in fp16 and its output is fp16
    "mxfp4_hw_f16_L1024": ("mxfp4_hw", "fp32", "c4", 1, 2, 1024, None, 128, "fp16"),
    "mxfp8_hw_f16_L1024": ("mxfp8_hw", "fp32", "c4", 1, 2, 1024, None, 128, "fp16"),
    "nvfp4_f16pv_L1024": ("nvfp4", "fp16_pv_only", "c5", 1, 2, 1024, None, 128, "fp16"),
    # the rest of the reference's config vocabulary (quant_config.py:199-346):
    # single-level, mixed-format, V-smoothed and E4M3-per-32 emulated configs,
    # and the two mixed hardware kernels (api.py:209-291)
    "mxfp4_s1_L512": ("mxfp4_s1", "fp32", "c4", 1, 1, 512, None),
    "mxfp8_s1_L512": ("mxfp8_s1", "fp32", "c4", 1, 1, 512, None),
    "mxfp4_s1_2level_L512": ("mxfp4_s1_2level", "fp32", "c4", 1, 1, 512, None),
    "mxfp4_s1_e4m3_L512": ("mxfp4_s1_e4m3", "fp32", "c4", 1, 1, 512, None),
    "mixed_fp8qk_fp4pv_L512": ("mixed_fp8qk_fp4pv", "fp32", "c4", 1, 1, 512, None),
    "mixed_fp4qk_fp8pv_L512": ("mixed_fp4qk_fp8pv", "fp32", "c4", 1, 1, 512, None),
    "mxfp4_s1_vsmooth_L512": ("mxfp4_s1_vsmooth", "fp32", "c4", 1, 1, 512, None),
    "mixed_fp8qk_fp4pv_vs_L512": ("mixed_fp8qk_fp4pv_vs", "fp32", "c4", 1, 1, 512, None),
    "mixed_fp4qk_fp8pv_vs_L512": ("mixed_fp4qk_fp8pv_vs", "fp32", "c4", 1, 1, 512, None),
    "mixed_mxfp8qk_mxfp4pv_hw_L512": ("mixed_mxfp8qk_mxfp4pv_hw", "fp32", "c4", 1, 1, 512, None),
    "mixed_mxfp4qk_mxfp8pv_hw_L512": ("mixed_mxfp4qk_mxfp8pv_hw", "fp32", "c4", 1, 1, 512, None),
}


def head_dim(name: str) -> int:
    return CASES[name][7] if len(CASES[name]) > 7 else 128


def input_dtype(name: str) -> torch.dtype:
    return torch.float16 if len(CASES[name]) > 8 and CASES[name][8] == "fp16" else torch.bfloat16


def case_inputs(name: str) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Seeded bf16 (or fp16) HND inputs [B, H, L, D] of a case (CPU, deterministic).

    c4: Q, V ~ N(0,1); K ~ N(0,1) + a per-(head, channel) offset ~ N(0, 3)
        shared by all tokens (BASELINE config 4's distribution).
    c5: Q, K, V ~ N(0,1); 1% of the K rows of every head scaled by 20
        (BASELINE config 5's distribution)."""
    _, _, dist, B, H, L, _ = CASES[name][:7]
    D = head_dim(name)
    seed = int(hashlib.sha256(name.encode()).hexdigest()[:8], 16)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, D, generator=g)
    k = torch.randn(B, H, L, D, generator=g)
    v = torch.randn(B, H, L, D, generator=g)
    if dist == "c4":
        k = k + torch.randn(B, H, 1, D, generator=g) * 3.0
    else:
        pick = torch.rand(B, H, L, 1, generator=g).argsort(dim=2) < max(1, L // 100)
        k = torch.where(pick, k * 20.0, k)
    dt = input_dtype(name)
    return q.to(dt), k.to(dt), v.to(dt)


def input_checksum(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in (q, k, v):
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def query_rows(name: str) -> np.ndarray:
    """Sequence positions of the query rows a case's fixture covers."""
    L, tiles = CASES[name][5], CASES[name][6]
    if tiles is None:
        return np.arange(L)
    return np.concatenate([np.arange(128 * t, min(L, 128 * t + 128)) for t in tiles])


# ---------------------------------------------------------------------------
# Triton interpreter gaps (this process only)
# ---------------------------------------------------------------------------
_E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def _bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def _f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).clamp(-448.0, 448.0)
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def _e4m3_to_f64(b: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(b, dtype=np.uint8)).view(torch.float8_e4m3fn) \
        .to(torch.float64).numpy()


def _e2m1_code_rne(x: np.ndarray) -> np.ndarray:
    """RNE onto E2M1 with saturation at 6 (cvt.rn.satfinite.e2m1x2.f32)."""
    x = np.asarray(x, np.float64)
    mag = np.minimum(np.abs(x), 6.0)
    grid = np.array([0, .5, 1, 1.5, 2, 3, 4, 6])
    hi = np.clip(np.searchsorted(grid, mag, side="left"), 0, 7)   # first grid value >= mag
    lo = np.clip(hi - 1, 0, 7)
    d_lo, d_hi = mag - grid[lo], grid[hi] - mag
    # nearer value wins; a tie goes to the even code (E2M1 codes: even = mantissa 0)
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    sign = (np.signbit(x) & ~np.isnan(x)).astype(np.uint8) << 3
    return code | sign


def install_interpreter_gaps() -> None:
    import triton.language as tl
    from triton._C.libtriton import ir
    from triton.language.semantic import TritonSemantic
    from triton.runtime import interpreter as I

    B = I.InterpreterBuilder
    TH = I.TensorHandle
    E2M1, E4M3 = ir.ScaleDotElemTypeTY.E2M1, ir.ScaleDotElemTypeTY.E4M3

    orig_semantic_dot_scaled = TritonSemantic.dot_scaled

    def semantic_dot_scaled(self, lhs, lhs_scale, lhs_format, rhs, rhs_scale, rhs_format, *rest, **kw):
        wrap = (lambda f: f if hasattr(f, "value") else tl.constexpr(f))
        return orig_semantic_dot_scaled(self, lhs, lhs_scale, wrap(lhs_format), rhs, rhs_scale,
                                        wrap(rhs_format), *rest, **kw)

    def decode(data, fmt, k_axis):
        if fmt == E2M1:
            lo, hi = _E2M1[data & 0xF], _E2M1[data >> 4]
            vals = np.stack([lo, hi], axis=k_axis + 1)
            shape = list(data.shape)
            shape[k_axis] *= 2
            return vals.reshape(shape)
        if fmt == E4M3:
            return _e4m3_to_f64(data)
        raise NotImplementedError(f"dot_scaled format {fmt}")

    def create_dot_scaled(self, lhs, lhs_scale, lhs_fmt, rhs, rhs_scale, rhs_fmt, fast_math,
                          lhs_k_pack, rhs_k_pack, acc):
        assert lhs_k_pack and rhs_k_pack
        a = decode(lhs.data, lhs_fmt, 1)           # [M, K]
        b = decode(rhs.data, rhs_fmt, 0)           # [K, N]
        if lhs_scale is not None:
            a = a * np.repeat(np.exp2(lhs_scale.data.astype(np.float64) - 127.0), 32, axis=1)
        if rhs_scale is not None:
            b = b * np.repeat(np.exp2(rhs_scale.data.astype(np.float64) - 127.0), 32, axis=1).T
        out = (acc.data.astype(np.float64) + a @ b).astype(np.float32)
        return TH(out, acc.dtype.scalar)

    class _AsmCall:
        def __init__(self, results):
            self.results = results

        def get_result(self, i):
            return self.results[i]

    def create_inline_asm(self, inline_asm, constraints, values, types, is_pure, pack):
        if "cvt.rn.satfinite.e2m1x2.f32" in inline_asm and len(values) == 2:
            hi, lo = values[0].data, values[1].data
            packed = (_e2m1_code_rne(hi).astype(np.uint32) << 4) | _e2m1_code_rne(lo).astype(np.uint32)
            ty = types[0]
            return _AsmCall([TH(packed.astype(np.uint32), getattr(ty, "scalar", ty))])
        raise NotImplementedError(f"inline asm not emulated: {inline_asm!r}")

    def is_bf16(h):
        return h.dtype.scalar == tl.bfloat16

    def as_f32(h):
        return _bf16_to_f32(h.data) if is_bf16(h) else h.data.astype(np.float32)

    orig_binary = B.binary_op

    def binary_op(self, lhs, rhs, op):
        if not (is_bf16(lhs) or is_bf16(rhs)):
            return orig_binary(self, lhs, rhs, op)
        out = op(as_f32(lhs), as_f32(rhs))
        if out.dtype == np.bool_:
            return TH(out, tl.int1)
        return TH(_f32_to_bf16(out), tl.bfloat16)

    orig_unary = B.unary_op

    def unary_op(self, arg, op):
        if not is_bf16(arg):
            return orig_unary(self, arg, op)
        return TH(_f32_to_bf16(op(_bf16_to_f32(arg.data))), tl.bfloat16)

    orig_fma = B.create_fma

    def create_fma(self, x, y, z):
        if not (is_bf16(x) or is_bf16(y) or is_bf16(z)):
            return orig_fma(self, x, y, z)
        return TH(_f32_to_bf16(as_f32(x) * as_f32(y) + as_f32(z)), tl.bfloat16)

    orig_dot = B.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if not (is_bf16(a) or is_bf16(b)):
            return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)
        out = as_f32(a).astype(np.float64) @ as_f32(b).astype(np.float64) + d.data.astype(np.float64)
        return TH(out.astype(np.float32), d.dtype.scalar)

    orig_cast = B.cast_impl

    def cast_impl(self, src, dst_type):
        s, t = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and t == tl.bfloat16:
            return TH(_f32_to_bf16(src.data), tl.bfloat16)
        if s == tl.bfloat16 and t == tl.float32:
            return TH(_bf16_to_f32(src.data), tl.float32)
        return orig_cast(self, src, dst_type)

    orig_fp_to_fp = B.create_fp_to_fp

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        s, t = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and t == tl.float8e4nv:
            return TH(_f32_to_e4m3(src.data), tl.float8e4nv)
        if s == tl.float32 and t == tl.bfloat16:
            return TH(_f32_to_bf16(src.data), tl.bfloat16)
        return orig_fp_to_fp(self, src, dst_type, rounding_mode)

    TritonSemantic.dot_scaled = semantic_dot_scaled
    B.create_dot_scaled = create_dot_scaled
    B.create_inline_asm = create_inline_asm
    B.binary_op = binary_op
    B.unary_op = unary_op
    B.create_fma = create_fma
    B.create_dot = create_dot
    B.cast_impl = cast_impl
    B.create_fp_to_fp = create_fp_to_fp
    # create_fadd, create_fmul, create_fcmp*, create_fp_trunc, ... are lambdas that
    # call self.binary_op / self.cast_impl, so they pick up the methods above.

    import triton

    class _CpuDriver:
        @staticmethod
        def get_active_torch_device():
            return torch.device("cpu")

    triton.runtime.driver.set_active(_CpuDriver())


def _self_check() -> None:
    """The E2M1 encoder against nearest-value rounding off the ties, and the
    tie rule; the bf16 rounding against torch's cast."""
    x = np.linspace(-7, 7, 20001)
    ties = np.isin(np.abs(x), [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    vals = _E2M1[_e2m1_code_rne(x)]
    nearest = np.abs(np.abs(x)[:, None] - _E2M1[None, :8]).argmin(axis=1)
    assert np.all((np.abs(vals) == _E2M1[nearest]) | ties | (np.abs(x) > 6))
    assert list(_E2M1[_e2m1_code_rne(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 9.0]))]) == \
        [0, 1, 1, 2, 2, 4, 4, 6]
    y = torch.randn(10000) * 100
    assert np.array_equal(_f32_to_bf16(y.numpy()), y.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


# ---------------------------------------------------------------------------
# running the reference
# ---------------------------------------------------------------------------
def run_case(name: str) -> np.ndarray:
    """The reference's output for a case, as bits of the input dtype [B, H, rows, D]."""
    config, acc, _, B, H, L, tiles = CASES[name][:7]
    from sage3 import api
    q, k, v = case_inputs(name)
    if tiles is None:
        out = api.sageattn3_standalone(q, k, v, config=config, acc_dtype=acc)
        return out.to(q.dtype).view(torch.int16).numpy().view(np.uint16)
    # Selected query tiles of the mxfp4_hw path: the steps of sage3/api.py:161-206
    # (smoothing over the whole sequence, padding, quantisation), then the
    # reference kernel on each chosen 128-row query tile with that tile's
    # delta_s row (the kernel reads delta_s row program_id(0)).
    assert config == "mxfp4_hw"
    import torch.nn.functional as F
    from sage3.mxfp4_hw_kernel import mxfp4_flash_attention, quantize_to_mxfp4
    from sage3.transforms import TransformContext, qk_smoothing
    qs, ks, vv, ctx = qk_smoothing(q, k, v, TransformContext())
    delta_s = ctx.delta_s
    pad = (128 - L % 128) % 128
    if pad:
        qs, ks, vv = (F.pad(t, (0, 0, 0, pad)) for t in (qs, ks, vv))
        delta_s = F.pad(delta_s, (0, pad))
    n = L + pad
    q_packed, q_scale = quantize_to_mxfp4(qs)
    k_packed, k_scale = quantize_to_mxfp4(ks)
    v_p, v_s = quantize_to_mxfp4(vv.permute(0, 1, 3, 2).contiguous().reshape(-1, n))
    v_packed, v_scale = v_p.reshape(B, H, 128, n // 2), v_s.reshape(B, H, 128, n // 32)
    outs = []
    for t in tiles:
        rows = slice(128 * t, 128 * t + 128)
        o = mxfp4_flash_attention(q_packed[:, :, rows], k_packed, v_packed, q_scale[:, :, rows], k_scale,
                                  v_scale, causal=False, sm_scale=1.0 / 128 ** 0.5,
                                  delta_s=delta_s[:, :, t:t + 1, :])
        outs.append(o[:, :, : min(L, 128 * t + 128) - 128 * t])
    out = torch.cat(outs, dim=2).to(torch.bfloat16)
    return out.view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path, help="checkout of the reference plugin")
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    _self_check()
    install_interpreter_gaps()
    sys.path.insert(0, str(args.reference / "src/vllm_qdq_plugin/sage3_attn"))
    out_path = HERE / "attn_reference.npz"
    data = dict(np.load(out_path)) if out_path.exists() else {}
    for name in args.only or list(CASES):
        t0 = time.time()
        q, k, v = case_inputs(name)
        data[f"{name}/out"] = run_case(name)
        data[f"{name}/checksum"] = np.array(input_checksum(q, k, v))
        data[f"{name}/rows"] = query_rows(name).astype(np.int32)
        print(f"{name}: {data[f'{name}/out'].shape} in {time.time() - t0:.1f} s", flush=True)
        np.savez_compressed(out_path, **data)
    print(f"wrote {out_path}")


if __name__ == "__main__":
    main()
