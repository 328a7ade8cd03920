"""GPU parity of the fused FP4 GEMMs with the very path they replace, run on
the same B200: the reference's activation QDQ followed by vLLM's compiled
Marlin kernels.

Reference path (what the plugin does today):
  dense  mxfp4_qdq(a) -> ops.marlin_gemm            (src/vllm_qdq_plugin/patch.py:51-57;
                                                      vllm/_custom_ops.py:1277)
  MoE    mxfp4_qdq(x) -> ops.moe_wna16_marlin_gemm   (patch.py:139-152; vllm/_custom_ops.py:2469)
Weights go through vLLM's own Marlin preparation
(vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py:205
prepare_fp4_layer_for_marlin, :522 prepare_moe_mxfp4_layer_for_marlin), whose
raw codes/scales this build captures for its own kernels.

The activation QDQ here is this build's kernel, which is bit-exact with the
reference's `mxfp4_qdq` (pinned by tests/golden/mxfp4_*.npz).  Every product
is exact in both GEMMs and both accumulate in fp32, so the outputs are
compared bit for bit, and, as a floor that holds whatever the summation
order, within bf16 output rounding plus an fp32-accumulation bound of the
exact product.
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from oracle import gemm as og

pytestmark = pytest.mark.gpu

REL = 2.0 ** -8
ACC = 2.0 ** -16


def _vllm():
    try:
        import vllm._custom_ops as ops
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
        from vllm.scalar_type import scalar_types
    except Exception as e:  # pragma: no cover - the GPU image ships vLLM
        pytest.skip(f"vLLM Marlin ops unavailable: {e}")
    return ops, mu, scalar_types


class _Layer(torch.nn.Module):
    pass


def _marlin_layer(codes: torch.Tensor, scales: torch.Tensor, n: int, k: int, dev):
    """A dense MXFP4 layer prepared by vLLM for Marlin (raw weights captured)."""
    from vllm_qdq_plugin import gemm
    _, mu, _ = _vllm()
    gemm.capture_marlin_weights()
    layer = _Layer()
    layer.weight = torch.nn.Parameter(codes.to(dev), requires_grad=False)
    layer.weight_scale = torch.nn.Parameter(scales.to(dev), requires_grad=False)
    layer.output_size_per_partition, layer.input_size_per_partition = n, k
    layer.params_dtype = torch.bfloat16
    layer.bias = None
    mu.prepare_fp4_layer_for_marlin(layer)
    return layer, gemm.lookup_marlin_weight(layer.weight)


def _within_exact(out: torch.Tensor, a: torch.Tensor, codes: np.ndarray, scales: np.ndarray, rows: int):
    exact, absum = og.qdq_linear_exact(a[:rows].view(torch.int16).numpy().view(np.uint16), codes, scales)
    got = out[:rows].float().cpu().numpy().astype(np.float64)
    return np.all(np.abs(got - exact) <= REL * np.abs(exact) + ACC * absum + 1e-30)


@pytest.mark.parametrize("m,n,k", [(1, 14336, 4096), (16, 14336, 4096), (256, 14336, 4096),
                                   (4096, 14336, 4096), (100, 768, 2048), (33, 512, 1024)])
def test_fused_linear_equals_qdq_plus_marlin(cuda_device, m, n, k):
    from vllm_qdq_plugin.gemm import mxfp4_linear
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    _, mu, _ = _vllm()
    rng = np.random.default_rng(m + n + k)
    codes = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = (127 + rng.integers(-10, -3, size=(n, k // 32))).astype(np.uint8)
    layer, w = _marlin_layer(torch.from_numpy(codes), torch.from_numpy(scales), n, k, cuda_device)
    assert w is not None, "prepare_fp4_layer_for_marlin was not captured"
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(m * 3 + k)).to(torch.bfloat16)
    ad = a.to(cuda_device)
    ref = mu.apply_fp4_marlin_linear(mxfp4_qdq(ad), layer.weight, layer.weight_scale, None,
                                     layer.workspace, n, k)
    ours = mxfp4_linear(ad, w)
    assert ours.shape == ref.shape and ours.dtype == ref.dtype
    assert _within_exact(ours, a, codes, scales, min(m, 64)), "fused linear outside the exact-product bound"
    assert _within_exact(ref, a, codes, scales, min(m, 64)), "Marlin outside the exact-product bound"
    diff = (ours.float() - ref.float()).abs()
    assert torch.equal(ours.view(torch.int16), ref.view(torch.int16)), (
        f"{int((diff > 0).sum())} of {diff.numel()} outputs differ from QDQ + Marlin, max {float(diff.max())}")


def test_patched_marlin_gemm_fused_route_equals_reference_route(cuda_device, monkeypatch):
    """The same patched `marlin_gemm` call, once down the reference route
    (QDQ, then the original Marlin op) and once down the fused route
    (VLLM_QDQ_FUSED_GEMM=1, captured weight): identical outputs."""
    from vllm_qdq_plugin import envs, patch
    from vllm_qdq_plugin.qdq import mxfp4_qdq, mxfp8_qdq
    ops, _, scalar_types = _vllm()
    n, k, m = 2048, 4096, 48
    rng = np.random.default_rng(11)
    codes = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = (127 + rng.integers(-10, -3, size=(n, k // 32))).astype(np.uint8)
    layer, _ = _marlin_layer(torch.from_numpy(codes), torch.from_numpy(scales), n, k, cuda_device)
    ns = types.SimpleNamespace(marlin_gemm=ops.marlin_gemm)
    patch._patch_marlin_gemm(ns, scalar_types, mxfp4_qdq, mxfp8_qdq, lambda *t: None)
    a = torch.randn(m, k, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(cuda_device)
    # the arguments vLLM's apply_fp4_marlin_linear passes (marlin_utils_fp4.py:149-202):
    # fp32 reduction of the split-K partial sums, no atomic add at this size
    args = (a, None, layer.weight, None, layer.weight_scale, None, None, None, None, None, layer.workspace,
            scalar_types.float4_e2m1f, m, n, k, True, False, True)
    monkeypatch.setenv("VLLM_QDQ_FUSED_GEMM", "0")
    ref = ns.marlin_gemm(*args)
    monkeypatch.setenv("VLLM_QDQ_FUSED_GEMM", "1")
    assert envs.VLLM_QDQ_FUSED_GEMM
    fused = ns.marlin_gemm(*args)
    assert torch.equal(fused.view(torch.int16), ref.view(torch.int16))


def test_grouped_moe_equals_qdq_plus_moe_marlin(cuda_device):
    """Grouped MXFP4 MoE GEMM vs mxfp4_qdq + moe_wna16_marlin_gemm on vLLM's
    own moe_align_block_size routing (w13-like layer, top-2 of 8 experts)."""
    from vllm.model_executor.layers.fused_moe.moe_align_block_size import moe_align_block_size
    from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_make_workspace_new

    from vllm_qdq_plugin import gemm
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    ops, mu, scalar_types = _vllm()
    gemm.capture_moe_weights()
    e, n2, k, m, top_k, bs = 8, 512, 1024, 96, 2, 16
    rng = np.random.default_rng(21)
    w13 = torch.from_numpy(rng.integers(0, 256, size=(e, n2, k // 2), dtype=np.uint8)).to(cuda_device)
    w13_s = torch.from_numpy((127 + rng.integers(-10, -3, size=(e, n2, k // 32))).astype(np.uint8)).to(cuda_device)
    w2 = torch.from_numpy(rng.integers(0, 256, size=(e, k, n2 // 4), dtype=np.uint8)).to(cuda_device)
    w2_s = torch.from_numpy((127 + rng.integers(-10, -3, size=(e, k, n2 // 64))).astype(np.uint8)).to(cuda_device)
    layer = _Layer()
    layer.params_dtype = torch.bfloat16
    mw13, mw2, mw13_s, _mw2_s, _, _ = mu.prepare_moe_mxfp4_layer_for_marlin(layer, w13, w2, w13_s, w2_s, None, None)
    captured = gemm._MOE_REGISTRY.get(mw13.data_ptr())
    assert captured is not None, "prepare_moe_mxfp4_layer_for_marlin was not captured"

    x = torch.randn(m, k, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(cuda_device)
    topk_ids = torch.from_numpy(np.argsort(rng.random((m, e)), axis=1)[:, :top_k].astype(np.int32)).to(cuda_device)
    topk_w = torch.rand(m, top_k, generator=torch.Generator().manual_seed(9)).to(cuda_device)
    sorted_ids, expert_ids, ntp = moe_align_block_size(topk_ids, bs, e)
    workspace = marlin_make_workspace_new(cuda_device, 4)
    ref = torch.zeros((m * top_k, n2), dtype=torch.bfloat16, device=cuda_device)
    ref = ops.moe_wna16_marlin_gemm(mxfp4_qdq(x), ref, mw13, None, mw13_s, None, None, None, None, None,
                                    workspace, sorted_ids, expert_ids, ntp, topk_w, moe_block_size=bs,
                                    top_k=top_k, mul_topk_weights=False, b_q_type=scalar_types.float4_e2m1f,
                                    size_m=m, size_n=n2, size_k=k, is_k_full=True, use_atomic_add=False,
                                    use_fp32_reduce=True, is_zp_float=False)
    ours = torch.zeros_like(ref)
    gemm.mxfp4_moe_linear(x, captured, sorted_ids, expert_ids, ntp, topk_w, bs, top_k, False, ours)
    # exact product per routed slot (bf16 output rounding + fp32 accumulation bound)
    ids = topk_ids.cpu().numpy()
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    got, want = ours.float().cpu().numpy(), ref.float().cpu().numpy()
    for ex in range(e):
        slots = np.nonzero(ids.reshape(-1) == ex)[0]
        exact, absum = og.qdq_linear_exact(xb[slots // top_k], w13[ex].cpu().numpy(), w13_s[ex].cpu().numpy())
        bound = REL * np.abs(exact) + ACC * absum + 1e-30
        assert np.all(np.abs(got[slots] - exact) <= bound), f"expert {ex}: grouped GEMM outside the bound"
        assert np.all(np.abs(want[slots] - exact) <= bound), f"expert {ex}: Marlin outside the bound"
    diff = np.abs(got - want)
    assert np.array_equal(ours.cpu().view(torch.int16).numpy(), ref.cpu().view(torch.int16).numpy()), (
        f"{int((diff > 0).sum())} of {diff.size} outputs differ from QDQ + moe_wna16_marlin_gemm, max {diff.max()}")
