"""GPU parity of the MXFP4 / NVFP4 / MXFP8 QDQ kernels (through the C ABI).

Bar: bit-exact against (a) the reference's own outputs in tests/golden/ and
(b) the pinned C oracle at larger, random, strided and odd shapes, including
the full BASELINE config-1 and config-2 tensors.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import qdq as oq

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "fp16": torch.float16}


def to_dev(bits: np.ndarray, tag: str, dev) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(DT[tag]).to(dev)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str):
    bad = np.argwhere(got != want)
    if len(bad):
        r, c = bad[0]
        raise AssertionError(f"{what}: {len(bad)} mismatches; first at {tuple(bad[0])}: "
                             f"got {got[r, c]:#06x} want {want[r, c]:#06x}")


# ------------------------------------------------------------------ golden
@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("subset", ["natural", "context", "c1_slice", "odd_k"])
def test_mxfp4_kernel_matches_reference_golden(cuda_device, tag, subset):
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    d = golden(f"mxfp4_{tag}.npz")
    y = mxfp4_qdq(to_dev(d[f"{subset}_x"], tag, cuda_device))
    assert_bits_equal(bits(y), d[f"{subset}_y"], f"mxfp4 {tag} {subset}")


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
def test_nvfp4_kernel_matches_reference_golden(cuda_device, tag):
    from vllm_qdq_plugin.qdq import nvfp4_qdq
    d = golden(f"nvfp4_{tag}.npz")
    for key in d.files:
        if not key.endswith("_y"):
            continue
        base = key[:-2]
        gs = d["c2_slice_gs"] if base == "c2_slice" else d["gs" + base.split("_gs")[1]]
        y = nvfp4_qdq(to_dev(d[base + "_x"], tag, cuda_device),
                      global_scale=torch.from_numpy(gs.astype(np.float32)).to(cuda_device))
        assert_bits_equal(bits(y), d[key], f"nvfp4 {tag} {base}")


# ------------------------------------------------------------------ oracle
def _random(m, k, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g) * torch.exp(torch.randn(m, 1, generator=g) * 3)
    x.view(-1)[torch.randperm(m * k, generator=g)[: max(1, m * k // 500)]] *= 64
    lim = torch.finfo(dtype).max / 4  # finite data: an inf amax makes every output NaN
    return x.clamp(-lim, lim).to(dtype).to(dev)


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 32), (3, 64), (257, 4096), (33, 96), (5, 100), (2, 7),
                                   (129, 1056)])
def test_mxfp4_kernel_matches_oracle(cuda_device, tag, shape):
    from vllm_qdq_plugin.qdq import mxfp4_qdq, mxfp4_quantize
    x = _random(*shape, DT[tag], seed=shape[0] * 7 + shape[1], dev=cuda_device)
    want, wcodes, wscales = oq.mxfp4_qdq(bits(x), fp16=(tag == "fp16"), codes=True)
    assert_bits_equal(bits(mxfp4_qdq(x)), want, f"mxfp4 {tag} {shape}")
    codes, scales = mxfp4_quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), wcodes)
    np.testing.assert_array_equal(scales.cpu().numpy(), wscales)


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 16), (3, 48), (257, 4096), (64, 8192), (7, 80)])
def test_nvfp4_kernel_matches_oracle(cuda_device, tag, shape):
    from vllm_qdq_plugin.qdq import nvfp4_global_scale, nvfp4_qdq, nvfp4_quantize
    x = _random(*shape, DT[tag], seed=shape[0] * 11 + shape[1], dev=cuda_device)
    gs_dev = nvfp4_global_scale(x)
    gs = oq.nvfp4_global_scale(bits(x), fp16=(tag == "fp16"))
    assert np.float32(gs_dev.item()) == np.float32(gs)
    want, wc, ws = oq.nvfp4_qdq(bits(x), gs, fp16=(tag == "fp16"), codes=True)
    assert_bits_equal(bits(nvfp4_qdq(x, global_scale=gs_dev)), want, f"nvfp4 {tag} {shape}")
    assert_bits_equal(bits(nvfp4_qdq(x)), want, f"nvfp4 auto-gs {tag} {shape}")
    codes, scales = nvfp4_quantize(x, gs_dev)
    np.testing.assert_array_equal(codes.cpu().numpy(), wc)
    np.testing.assert_array_equal(scales.cpu().numpy(), ws)


def test_strided_rows_and_unaligned_views(cuda_device):
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq
    base = _random(64, 4096 + 64, torch.bfloat16, seed=5, dev=cuda_device)
    for view in (base[:, :4096], base[:, 8:8 + 4096 - 32], base[1:, 3:3 + 1024]):
        want = oq.mxfp4_qdq(bits(view))
        assert_bits_equal(bits(mxfp4_qdq(view)), want, f"mxfp4 view {tuple(view.stride())}")
        if view.shape[1] % 16 == 0:
            gs = torch.tensor([3.0], device=cuda_device)
            assert_bits_equal(bits(nvfp4_qdq(view, global_scale=gs)),
                              oq.nvfp4_qdq(bits(view), 3.0), "nvfp4 view")
    t = base.t()  # column-major: made contiguous by the wrapper
    assert_bits_equal(bits(mxfp4_qdq(t)), oq.mxfp4_qdq(bits(t)), "transposed")


def test_empty_and_special_values(cuda_device):
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq
    assert mxfp4_qdq(torch.empty(0, 64, dtype=torch.bfloat16, device=cuda_device)).shape == (0, 64)
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda_device)
    x[1] = -0.0
    x[2, 5] = float("inf")
    x[2, 6] = -3.0
    x[3, :32] = torch.finfo(torch.bfloat16).max
    assert_bits_equal(bits(mxfp4_qdq(x)), oq.mxfp4_qdq(bits(x)), "specials mxfp4")
    gs = torch.tensor([2.5], device=cuda_device)
    assert_bits_equal(bits(nvfp4_qdq(x, global_scale=gs)), oq.nvfp4_qdq(bits(x), 2.5),
                      "specials nvfp4")


# ------------------------------------------------------------------ MXFP8
@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("subset", ["natural", "context", "c1_slice", "odd_k"])
def test_mxfp8_kernel_matches_reference_golden(cuda_device, tag, subset):
    from vllm_qdq_plugin.qdq import mxfp8_qdq
    d = golden(f"mxfp8_{tag}.npz")
    y = mxfp8_qdq(to_dev(d[f"{subset}_x"], tag, cuda_device))
    assert_bits_equal(bits(y), d[f"{subset}_y"], f"mxfp8 {tag} {subset}")


@pytest.mark.parametrize("tag", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 32), (3, 64), (257, 4096), (33, 96), (5, 100), (2, 7),
                                   (129, 1056)])
def test_mxfp8_kernel_matches_oracle(cuda_device, tag, shape):
    from vllm_qdq_plugin.qdq import mxfp8_qdq, mxfp8_quantize
    x = _random(*shape, DT[tag], seed=shape[0] * 13 + shape[1], dev=cuda_device)
    want, wcodes, wscales = oq.mxfp8_qdq(bits(x), fp16=(tag == "fp16"), codes=True)
    assert_bits_equal(bits(mxfp8_qdq(x)), want, f"mxfp8 {tag} {shape}")
    codes, scales = mxfp8_quantize(x)
    k = shape[1]
    np.testing.assert_array_equal(codes.cpu().numpy()[:, :k], wcodes)
    assert not codes.cpu().numpy()[:, k:].any()  # zero padding up to a multiple of 32
    np.testing.assert_array_equal(scales.cpu().numpy(), wscales)


def test_mxfp8_specials_strides_and_underflow(cuda_device):
    """Zeros of both signs, inf, the largest values, E4M3's subnormal range and
    bf16 groups whose max is so large that small elements underflow to zero
    when divided by the scale (they come out +0, as torch.sign(-0) is 0)."""
    from vllm_qdq_plugin.qdq import mxfp8_qdq
    x = torch.zeros(6, 64, dtype=torch.bfloat16)
    x[1] = -0.0
    x[2, 5] = float("inf")
    x[2, 6] = -3.0
    x[3, :32] = torch.finfo(torch.bfloat16).max
    x[4, 0] = 2.0 ** 100
    x[4, 1:32] = -torch.exp2(-torch.arange(100, 131).float())
    x[4, 32] = -(2.0 ** 40)
    x[4, 33:64] = torch.exp2(-torch.arange(100, 131).float()) * torch.tensor(
        [(-1) ** i for i in range(31)]).float()
    x[5] = torch.linspace(-1, 1, 64) * 2.0 ** -8
    x[5, 0] = 1.0
    xd = x.to(cuda_device)
    assert_bits_equal(bits(mxfp8_qdq(xd)), oq.mxfp8_qdq(bits(x)), "mxfp8 specials")
    base = _random(64, 4096 + 64, torch.bfloat16, seed=15, dev=cuda_device)
    for view in (base[:, :4096], base[:, 8:8 + 4096 - 32], base[1:, 3:3 + 1000]):
        assert_bits_equal(bits(mxfp8_qdq(view)), oq.mxfp8_qdq(bits(view)), f"mxfp8 view {tuple(view.stride())}")
    assert mxfp8_qdq(torch.empty(0, 64, dtype=torch.float16, device=cuda_device)).shape == (0, 64)


def test_mxfp8_config1_shape_bit_exact_and_idempotent(cuda_device):
    from bench import c1_input
    from vllm_qdq_plugin.qdq import mxfp8_qdq
    x = c1_input()
    y = mxfp8_qdq(x.to(cuda_device))
    want = oq.mxfp8_qdq(bits(x))
    assert_bits_equal(bits(y), want, "mxfp8 config-1 shape")
    # A second pass keeps every value (they are on the E4M3 grid of the same
    # scales) but, like the reference, turns the -0 of tiny negative inputs
    # into +0 (torch.sign(-0) is 0): equal as floats, and bit-exact with the
    # oracle's second pass.
    y2 = mxfp8_qdq(y)
    assert torch.equal(y2.float(), y.float())
    assert_bits_equal(bits(y2), oq.mxfp8_qdq(want), "mxfp8 second pass")


# ------------------------------------------------------------------ full size
def test_config1_full_size_bit_exact_and_idempotent(cuda_device):
    from bench import c1_input
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    x = c1_input()
    y = mxfp4_qdq(x.to(cuda_device))
    assert_bits_equal(bits(y), oq.mxfp4_qdq(bits(x)), "config 1 full")
    # QDQ'd activations are exactly MXFP4-representable: a second pass is a no-op
    assert torch.equal(mxfp4_qdq(y).view(torch.int16), y.view(torch.int16))


def test_config2_full_size_bit_exact(cuda_device):
    from bench import c2_input, global_scale_of
    from vllm_qdq_plugin.qdq import nvfp4_global_scale, nvfp4_qdq
    x = c2_input()
    gs = global_scale_of(x)
    xd = x.to(cuda_device)
    assert np.float32(nvfp4_global_scale(xd).item()) == np.float32(gs.item())
    y = nvfp4_qdq(xd, global_scale=gs.to(cuda_device))
    assert_bits_equal(bits(y), oq.nvfp4_qdq(bits(x), float(gs)), "config 2 full")


def test_ops_trace_under_torch_compile(cuda_device):
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq

    def f(a, gs):
        return mxfp4_qdq(a * 2) + nvfp4_qdq(a, global_scale=gs)

    a = _random(64, 256, torch.bfloat16, seed=9, dev=cuda_device)
    gs = torch.tensor([1.5], device=cuda_device)
    eager = f(a, gs)
    compiled = torch.compile(f, fullgraph=True)(a, gs)
    assert torch.equal(eager.view(torch.int16), compiled.view(torch.int16))


def test_nvfp4_activation_knob_end_to_end(cuda_device):
    """VLLM_QDQ_NVFP4_ACT=1 on an NVFP4 Marlin layer: the activation reaching the
    (stand-in) Marlin kernel is exactly nvfp4_qdq(a) with a's own global scale."""
    import os
    import types
    from unittest import mock

    from vllm_qdq_plugin import patch as P
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq
    st = types.SimpleNamespace(float4_e2m1f=object(), float8_e4m3fn=object())
    ops = types.SimpleNamespace(marlin_gemm=lambda *a, **k: a[0])
    P._patch_marlin_gemm(ops, st, mxfp4_qdq, None, lambda *t: None)
    a = _random(64, 4096, torch.bfloat16, seed=77, dev=cuda_device)
    with mock.patch.dict(os.environ, {"VLLM_QDQ_NVFP4_ACT": "1"}):
        got = ops.marlin_gemm(a, None, None, None, None, None, torch.ones(1, device=cuda_device), None,
                              None, None, None, st.float4_e2m1f, 64, 8, 4096)
    assert_bits_equal(bits(got), bits(nvfp4_qdq(a)), "NVFP4 activation knob")
    gs = oq.nvfp4_global_scale(bits(a))
    assert_bits_equal(bits(got), oq.nvfp4_qdq(bits(a), gs), "NVFP4 activation knob vs oracle")


# ------------------------------------------------------------------ host-resident input
@pytest.mark.parametrize("fmt", ["mxfp4", "mxfp8", "nvfp4"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_streamed_host_qdq_equals_device_qdq(cuda_device, fmt, dtype):
    """Row blocks streamed through the GPU (H2D, QDQ and D2H on three streams)
    give the device hook's output bit for bit: ragged last block, more blocks
    than staging slots, pinned and pageable outputs, and back-to-back calls."""
    from vllm_qdq_plugin.qdq import mxfp4_qdq, mxfp8_qdq, nvfp4_qdq, qdq_from_host
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(1000, 256, generator=g) * torch.exp(torch.randn(1000, 1, generator=g) * 3)).to(dtype)
    xd = x.to(cuda_device)
    gs = torch.tensor([2688.0], dtype=torch.float32) / x.float().abs().max()
    if fmt == "nvfp4":
        want = nvfp4_qdq(xd, global_scale=gs.to(cuda_device))
    else:
        want = (mxfp4_qdq if fmt == "mxfp4" else mxfp8_qdq)(xd)
    want = bits(want)
    kw = dict(global_scale=gs) if fmt == "nvfp4" else {}
    got = qdq_from_host(x.pin_memory(), fmt, block_bytes=37 * 256 * 2, depth=3, **kw)
    assert got.is_pinned()
    assert_bits_equal(bits(got), want, f"{fmt} streamed, pinned out")
    out = torch.empty_like(x)
    qdq_from_host(x, fmt, out=out, block_bytes=300 * 256 * 2, depth=2, **kw)
    assert_bits_equal(bits(out), want, f"{fmt} streamed, pageable")
    again = qdq_from_host(x.pin_memory(), fmt, non_blocking=True, **kw)
    torch.cuda.current_stream(cuda_device).synchronize()
    assert_bits_equal(bits(again), want, f"{fmt} streamed, one block")
