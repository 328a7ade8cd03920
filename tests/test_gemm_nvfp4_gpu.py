"""GPU parity of the NVFP4 fused linear (tcgen05 kind::mxf4nvf4, block16).

What it replaces, on NVFP4 Marlin layers with VLLM_QDQ_NVFP4_ACT=1:
  nvfp4_qdq(a) -> vLLM marlin_gemm with the layer's E4M3 scales and tensor scale
  (vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py:149-202,
  vllm/_custom_ops.py:1277).  The activation codes and scales are the ones
  nvfp4_qdq emits (bit-exact with vLLM's ref_nvfp4_quant, tests/golden/nvfp4_*.npz).

Tolerances (exact = float64 product of the unrounded dequantised operands,
absum = sum |a_k w_k|):
  fused vs exact         2^-8 |exact| + 2^-16 absum   (bf16 output rounding +
                                                       fp32 accumulation)
  fused vs QDQ + Marlin  2^-8 |exact| + (2^-9 + 2^-15) absum   (nvfp4_qdq rounds
                         every activation element to bf16, a relative 2^-9)
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import qdq as oq

pytestmark = pytest.mark.gpu

REL = 2.0 ** -8
ACC = 2.0 ** -16


def _weight(n, k, seed, dev):
    from vllm_qdq_plugin.gemm import prepare_nvfp4_weight
    codes, scales, gs = og.random_nvfp4_weight(n, k, seed)
    w = prepare_nvfp4_weight(torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev), gs)
    return w, codes, scales, gs


def _bad(got: torch.Tensor, want: np.ndarray, exact: np.ndarray, absum: np.ndarray, acc: float) -> int:
    g = got.float().cpu().numpy().astype(np.float64)
    return int((np.abs(g - want) > REL * np.abs(exact) + acc * absum + 1e-30).sum())


# M <= 64 runs the swap-AB decode kernel (activation quantised in its producer),
# larger M the block16 GEMM after a separate quantisation pass
@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (1, 1024, 4096), (16, 512, 4096), (300, 768, 2048),
                                   (129, 257, 288), (512, 1024, 4096), (5, 384, 2080), (33, 256, 512),
                                   (64, 640, 1024), (17, 14336, 4096)])
def test_nvfp4_linear_matches_exact(cuda_device, m, n, k):
    from vllm_qdq_plugin.gemm import nvfp4_linear
    w, codes, scales, gs = _weight(n, k, m + n + k, cuda_device)
    a = (torch.randn(m, k, generator=torch.Generator().manual_seed(m * 7 + k)) *
         torch.exp(torch.randn(m, 1, generator=torch.Generator().manual_seed(m)))).to(torch.bfloat16)
    out = nvfp4_linear(a.to(cuda_device), w)
    assert out.shape == (m, n) and out.dtype == torch.bfloat16
    exact, _, absum = og.nvfp4_linear_exact(a.view(torch.int16).numpy().view(np.uint16), codes, scales, gs)
    assert _bad(out, exact, exact, absum, ACC) == 0
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


# The activation's global scale inside the call comes from the GEMM path's
# multi-CTA pass (M > 64), or for M <= 64 from the decode kernel's clusters of
# 4 CTAs (M <= 24 and N / 128 a multiple of 4: n = 1024) or a separate 8-CTA
# cluster pass; all must equal nvfp4_global_scale bit for bit.
@pytest.mark.parametrize("n", [384, 1024])
@pytest.mark.parametrize("m,k", [(200, 1024), (64, 1024), (24, 1024), (9, 2080), (8, 1024), (3, 288)])
def test_nvfp4_linear_fp16_bias_and_given_global_scale(cuda_device, m, k, n):
    from vllm_qdq_plugin.gemm import nvfp4_linear
    from vllm_qdq_plugin.qdq import nvfp4_global_scale
    w, codes, scales, gs = _weight(n, k, 3, cuda_device)
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(1)).to(torch.float16)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(2)).to(torch.float16)
    ad = a.to(cuda_device)
    gs_a = nvfp4_global_scale(ad)
    out = nvfp4_linear(ad, w, bias=bias.to(cuda_device), a_global_scale=gs_a)
    assert out.dtype == torch.float16
    exact, _, absum = og.nvfp4_linear_exact(a.view(torch.int16).numpy().view(np.uint16), codes, scales, gs,
                                             fp16=True, a_global_scale=float(gs_a.item()))
    exact = exact + bias.double().numpy()[None, :]
    assert _bad(out, exact, exact, absum, ACC) == 0
    # computing gs_a inside the call gives the same result
    assert torch.equal(nvfp4_linear(ad, w, bias=bias.to(cuda_device)).view(torch.int16), out.view(torch.int16))


class _Layer(torch.nn.Module):
    pass


def _nvfp4_marlin_layer(codes, scales, gs, n, k, dev):
    from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu

    from vllm_qdq_plugin import gemm
    gemm.capture_marlin_weights()
    layer = _Layer()
    layer.weight = torch.nn.Parameter(torch.from_numpy(codes).to(dev), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(torch.from_numpy(scales).to(dev).view(torch.float8_e4m3fn),
                                            requires_grad=False)
    layer.weight_global_scale = torch.nn.Parameter(torch.tensor(gs, dtype=torch.float32, device=dev),
                                                   requires_grad=False)
    layer.output_size_per_partition, layer.input_size_per_partition = n, k
    layer.params_dtype, layer.bias = torch.bfloat16, None
    mu.prepare_fp4_layer_for_marlin(layer)
    return layer, gemm.lookup_marlin_weight(layer.weight), mu


@pytest.mark.parametrize("m", [16, 4096])
def test_nvfp4_linear_vs_nvfp4_qdq_plus_marlin(cuda_device, m):
    """Same box, same weights: vLLM's own Marlin NVFP4 path on nvfp4_qdq(a)."""
    pytest.importorskip("vllm._custom_ops")
    from vllm_qdq_plugin.gemm import Nvfp4Weight, nvfp4_linear
    from vllm_qdq_plugin.qdq import nvfp4_qdq
    n, k = 2048, 4096
    codes, scales, gs = og.random_nvfp4_weight(n, k, 77)
    layer, w, mu = _nvfp4_marlin_layer(codes, scales, gs, n, k, cuda_device)
    assert isinstance(w, Nvfp4Weight) and w.global_scale == gs
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    ad = a.to(cuda_device)
    ref = mu.apply_fp4_marlin_linear(nvfp4_qdq(ad), layer.weight, layer.weight_scale, layer.weight_global_scale,
                                     layer.workspace, n, k)
    ours = nvfp4_linear(ad, w)
    rows = min(m, 64)
    # the activation's global scale is over all M rows, as nvfp4_qdq computes it
    gs_a = oq.nvfp4_global_scale(a.view(torch.int16).numpy().view(np.uint16))
    exact, via_qdq, absum = og.nvfp4_linear_exact(a[:rows].view(torch.int16).numpy().view(np.uint16),
                                                   codes, scales, gs, a_global_scale=gs_a)
    # Marlin reproduces the QDQ'd product; the fused linear the unrounded one; the two agree
    assert _bad(ref[:rows], via_qdq, via_qdq, absum, ACC) == 0
    assert _bad(ours[:rows], exact, exact, absum, ACC) == 0
    assert _bad(ours[:rows], ref[:rows].float().cpu().numpy().astype(np.float64), exact, absum,
                2.0 ** -9 + 2.0 ** -15) == 0
    rel = float((ours.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 4e-3, rel


def test_patched_marlin_gemm_routes_nvfp4_layers(cuda_device, monkeypatch):
    """The patched marlin_gemm on an NVFP4 layer: with VLLM_QDQ_FUSED_GEMM=1
    and VLLM_QDQ_NVFP4_ACT=1 it runs the NVFP4 fused linear (close to the
    NVFP4 QDQ + Marlin route); without VLLM_QDQ_NVFP4_ACT it keeps the
    reference route (MXFP4 QDQ + Marlin) bit for bit."""
    pytest.importorskip("vllm._custom_ops")
    import vllm._custom_ops as ops
    from vllm.scalar_type import scalar_types

    from vllm_qdq_plugin import patch
    from vllm_qdq_plugin.qdq import mxfp4_qdq, mxfp8_qdq
    n, k, m = 1024, 2048, 40
    codes, scales, gs = og.random_nvfp4_weight(n, k, 5)
    layer, _, _ = _nvfp4_marlin_layer(codes, scales, gs, n, k, cuda_device)
    ns = types.SimpleNamespace(marlin_gemm=ops.marlin_gemm)
    patch._patch_marlin_gemm(ns, scalar_types, mxfp4_qdq, mxfp8_qdq, lambda *t: None)
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(cuda_device)
    args = (a, None, layer.weight, None, layer.weight_scale, None, layer.weight_global_scale, None, None, None,
            layer.workspace, scalar_types.float4_e2m1f, m, n, k, True, False, True)
    monkeypatch.setenv("VLLM_QDQ_NVFP4_ACT", "1")
    monkeypatch.setenv("VLLM_QDQ_FUSED_GEMM", "0")
    ref_nv = ns.marlin_gemm(*args)
    monkeypatch.setenv("VLLM_QDQ_FUSED_GEMM", "1")
    fused = ns.marlin_gemm(*args)
    assert float((fused.float() - ref_nv.float()).norm() / ref_nv.float().norm()) < 4e-3
    monkeypatch.setenv("VLLM_QDQ_NVFP4_ACT", "0")
    ref_mx = ns.marlin_gemm(*args)
    monkeypatch.setenv("VLLM_QDQ_FUSED_GEMM", "0")
    assert torch.equal(ref_mx.view(torch.int16), ns.marlin_gemm(*args).view(torch.int16))
