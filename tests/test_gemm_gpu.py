"""GPU parity of the tcgen05 block-scaled MXFP4 GEMM (through the C ABI).

Reference semantics: mxfp4_qdq(a) then Marlin's bf16 x dequantised-MXFP4 GEMM
with fp32 accumulation (src/vllm_qdq_plugin/patch.py:57 + vllm/_custom_ops.py:1277).
Every product is exact in both, so the tolerance is the output rounding
(2^-8 relative, bf16) plus an fp32-accumulation bound of 2^-16 x sum|a_k w_k|.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import qdq as oq

pytestmark = pytest.mark.gpu

REL = 2.0 ** -8
ACC = 2.0 ** -16


def _check(out: torch.Tensor, exact: np.ndarray, absum: np.ndarray, what: str):
    got = out.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - exact)
    bound = REL * np.abs(exact) + ACC * absum + 1e-30
    bad = err > bound
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside tolerance; first {tuple(i)} "
                             f"got {got[tuple(i)]} want {exact[tuple(i)]} bound {bound[tuple(i)]}")


def _inputs(m, n, k, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dtype)
    codes, scales = og.random_mxfp4_weight(n, k, seed + 1)
    return a, codes, scales


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (256, 512, 1024), (100, 300, 512),
                                   (1, 256, 4096), (16, 512, 4096), (333, 768, 2048),
                                   (129, 257, 288)])
def test_fused_linear_matches_qdq_marlin_oracle(cuda_device, m, n, k):
    from vllm_qdq_plugin.gemm import mxfp4_linear, prepare_mxfp4_weight
    a, codes, scales = _inputs(m, n, k, seed=m * 31 + n + k)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    out = mxfp4_linear(a.to(cuda_device), w)
    assert out.dtype == torch.bfloat16 and out.shape == (m, n)
    abits = a.view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales)
    _check(out, exact, absum, f"linear {m}x{n}x{k}")


@pytest.mark.parametrize("m,n,k", [(1, 14336, 4096), (3, 300, 4128), (17, 512, 1024), (33, 640, 512),
                                   (64, 1024, 2048)])
def test_decode_path_matches_oracle(cuda_device, m, n, k):
    """M <= 64 runs the one-launch kernel that quantises the activation inside
    the GEMM producer (swap-AB tcgen05 MMAs, W rows on the M side)."""
    from vllm_qdq_plugin.gemm import mxfp4_linear, prepare_mxfp4_weight
    a, codes, scales = _inputs(m, n, k, seed=m * 7 + n + k)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    out = mxfp4_linear(a.to(cuda_device), w)
    abits = a.view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales)
    _check(out, exact, absum, f"decode {m}x{n}x{k}")
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


def test_decode_path_fp16_bias_and_codes_path(cuda_device):
    """fp16 activation with bias on the decode path, and agreement with the
    three-launch path (QDQ codes -> tiled scales -> GEMM) within the fp32
    accumulation bound."""
    from vllm_qdq_plugin.gemm import mxfp4_gemm_codes, mxfp4_linear, prepare_mxfp4_weight
    from vllm_qdq_plugin.qdq import mxfp4_quantize
    m, n, k = 5, 384, 1024
    a, codes, scales = _inputs(m, n, k, seed=9, dtype=torch.float16)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(10)).to(torch.float16)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    out = mxfp4_linear(a.to(cuda_device), w, bias.to(cuda_device))
    abits = a.view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales, bias.float().numpy(), fp16=True)
    _check(out, exact, absum + np.abs(bias.float().numpy())[None, :], "decode fp16 + bias")
    ab, _, _ = _inputs(m, n, k, seed=9)
    ad = ab.to(cuda_device)
    ac, asf = mxfp4_quantize(ad)
    ref = mxfp4_gemm_codes(ac, asf, w).float().cpu().numpy().astype(np.float64)
    exact_b, absum_b = og.qdq_linear_exact(ab.view(torch.int16).numpy().view(np.uint16), codes, scales)
    got = mxfp4_linear(ad, w).float().cpu().numpy().astype(np.float64)
    assert (np.abs(got - ref) <= 2 * (REL * np.abs(exact_b) + ACC * absum_b) + 1e-30).all()


def test_fp16_activation_and_bias(cuda_device):
    from vllm_qdq_plugin.gemm import mxfp4_linear, prepare_mxfp4_weight
    m, n, k = 200, 512, 1024
    a, codes, scales = _inputs(m, n, k, seed=3, dtype=torch.float16)
    bias = torch.randn(n, generator=torch.Generator().manual_seed(4)).to(torch.float16)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    out = mxfp4_linear(a.to(cuda_device), w, bias.to(cuda_device))
    assert out.dtype == torch.float16
    abits = a.view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales, bias.float().numpy(), fp16=True)
    _check(out, exact, absum + np.abs(bias.float().numpy())[None, :], "fp16 + bias")


def test_codes_path_equals_fused_path(cuda_device):
    from vllm_qdq_plugin.gemm import mxfp4_gemm_codes, mxfp4_linear, prepare_mxfp4_weight
    from vllm_qdq_plugin.qdq import mxfp4_quantize
    m, n, k = 256, 1024, 2048
    a, codes, scales = _inputs(m, n, k, seed=11)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    ad = a.to(cuda_device)
    ac, asf = mxfp4_quantize(ad)
    assert torch.equal(mxfp4_gemm_codes(ac, asf, w), mxfp4_linear(ad, w))


def test_config3_full_size_rows_and_row_independence(cuda_device):
    """M=4096, N=14336, K=4096; a row sample is checked against
    the oracle, and every row must equal the same row computed alone (M=1)."""
    from vllm_qdq_plugin.gemm import mxfp4_linear, prepare_mxfp4_weight
    m, n, k = 4096, 14336, 4096
    g = torch.Generator().manual_seed(2)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    codes, scales = og.random_mxfp4_weight(n, k, seed=3)
    w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                             torch.from_numpy(scales).to(cuda_device))
    ad = a.to(cuda_device)
    out = mxfp4_linear(ad, w)
    rows = np.array([0, 1, 127, 128, 2047, 4000, 4095])
    abits = a[rows].contiguous().view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales)
    _check(out[rows], exact, absum, "config 3 rows")
    for r in (0, 4095):
        single = mxfp4_linear(ad[r:r + 1], w)
        assert torch.equal(single[0], out[r])
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


def test_marlin_hook_routes_captured_layers(cuda_device):
    import types
    from vllm_qdq_plugin import gemm, patch
    m, n, k = 64, 256, 512
    a, codes, scales = _inputs(m, n, k, seed=21)
    marlin_weight = torch.zeros(8, dtype=torch.int32, device=cuda_device)  # stands for the repacked weight
    w = gemm.prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                                  torch.from_numpy(scales).to(cuda_device))
    gemm.register_marlin_weight(marlin_weight, w)
    st = types.SimpleNamespace(float4_e2m1f=object(), float8_e4m3fn=object())
    ops = types.SimpleNamespace(marlin_gemm=lambda *args: (_ for _ in ()).throw(AssertionError("Marlin called")))
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    patch._patch_marlin_gemm(ops, st, mxfp4_qdq, None, lambda *t: None)
    import os
    from unittest import mock
    with mock.patch.dict(os.environ, {"VLLM_QDQ_FUSED_GEMM": "1"}):
        out = ops.marlin_gemm(a.to(cuda_device), None, marlin_weight, None, torch.empty(1), None, None,
                              None, None, None, torch.empty(1), st.float4_e2m1f, m, n, k)
    abits = a.view(torch.int16).numpy().view(np.uint16)
    exact, absum = og.qdq_linear_exact(abits, codes, scales)
    _check(out, exact, absum, "hook")


# ------------------------------------------------------------------ grouped MoE GEMM
def _moe_case(m, e, top_k, bs, n, k, seed, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dtype)
    ws = [og.random_mxfp4_weight(n, k, seed * 31 + i) for i in range(e)]
    codes = np.stack([c for c, _ in ws])
    scales = np.stack([s for _, s in ws])
    topk_ids = np.stack([rng.permutation(e)[:top_k] for _ in range(m)])  # distinct experts per token
    sorted_ids, expert_ids, ntp = og.moe_align(topk_ids, e, bs)
    topk_w = rng.random((m, top_k)).astype(np.float32)
    return a, codes, scales, sorted_ids, expert_ids, ntp, topk_w


@pytest.mark.parametrize("m,e,top_k,bs,n,k,mul", [(5, 4, 2, 16, 256, 512, False),
                                                  (37, 8, 2, 16, 384, 1024, True),
                                                  (64, 16, 4, 32, 200, 2048, True),
                                                  (3, 4, 1, 64, 128, 288, False),
                                                  (100, 8, 8, 8, 256, 512, True),
                                                  (300, 6, 2, 64, 384, 1024, True),
                                                  (2048, 4, 2, 8, 128, 256, False),
                                                  (512, 4, 2, 64, 320, 512, True),
                                                  (150, 4, 2, 48, 256, 512, False)])
def test_moe_grouped_gemm_matches_oracle(cuda_device, m, e, top_k, bs, n, k, mul):
    """Grouped MXFP4 MoE GEMM (the reference's mxfp4_qdq + moe_wna16_marlin_gemm)
    on vLLM's moe_align_block_size layout: every routed slot's row against the
    exact oracle, with the fused GEMM's tolerance.  The cases cover one block
    per expert, runs of 2 and 13 blocks (cut into segments of at most 3), a
    1024-block layout whose runs cross the segment scan's 256-block chunks,
    three-block segments of 64 rows (one MMA with N = 192), and a block size
    (48) below the kernel's 64-row block tile."""
    from vllm_qdq_plugin.gemm import mxfp4_moe_linear, prepare_mxfp4_moe_weight
    a, codes, scales, sid, eid, ntp, topk_w = _moe_case(m, e, top_k, bs, n, k, seed=m + e + bs)
    dev = cuda_device
    w = prepare_mxfp4_moe_weight(torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev))
    out = mxfp4_moe_linear(a.to(dev), w, torch.from_numpy(sid).to(dev), torch.from_numpy(eid).to(dev),
                           torch.from_numpy(ntp).to(dev), torch.from_numpy(topk_w).to(dev), bs, top_k, mul)
    rows = og.moe_linear_exact(a.view(torch.int16).numpy().view(np.uint16), codes, scales, sid, eid,
                               int(ntp[0]), bs, top_k, topk_w.reshape(-1) if mul else None)
    assert len(rows) == m * top_k
    got = out.float().cpu().numpy()
    slots = np.array(sorted(rows))
    exact = np.stack([rows[s][0] for s in slots])
    absum = np.stack([rows[s][1] for s in slots])
    _check(torch.from_numpy(got[slots]), exact, absum, f"moe m={m} e={e} top_k={top_k} bs={bs}")
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


@pytest.mark.parametrize("k", [288, 2880])
def test_moe_result_independent_of_stale_workspace(cuda_device, k):
    """K not a multiple of 256: the GEMM's last K stage reads scale bytes past
    K / 32, which the pre-pass writes as E8M0 0.  A workspace left full of
    0xFF (NaN scales) by earlier use must give the bit-identical result."""
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.gemm import prepare_mxfp4_moe_weight
    m, e, top_k, bs, n = 40, 4, 2, 16, 256
    a, codes, scales, sid, eid, ntp, topk_w = _moe_case(m, e, top_k, bs, n, k, seed=k)
    dev = cuda_device
    w = prepare_mxfp4_moe_weight(torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev))
    ad, sidd, eidd, ntpd, twd = (t.to(dev) for t in (a, torch.from_numpy(sid), torch.from_numpy(eid),
                                                     torch.from_numpy(ntp), torch.from_numpy(topk_w).reshape(-1)))
    lib = _native.lib()
    outs = []
    for fill in (0x00, 0xFF):
        ws = torch.full((lib.fp4_moe_workspace_bytes(sidd.numel(), bs, k),), fill, dtype=torch.uint8, device=dev)
        out = torch.zeros((m * top_k, n), dtype=torch.bfloat16, device=dev)
        _native.check("fp4_moe_mxf4", lib.fp4_moe_mxf4(
            ad.data_ptr(), k, 0, w.codes.data_ptr(), w.sf_tiled.data_ptr(), e, sidd.data_ptr(), eidd.data_ptr(),
            ntpd.data_ptr(), twd.data_ptr(), sidd.numel(), bs, top_k, 1, out.data_ptr(), n, m, n, k,
            ws.data_ptr(), ws.numel(), _native.stream_ptr(dev)))
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.isfinite(outs[1].float()).all()
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))


def test_moe_skips_foreign_experts_and_padding_blocks(cuda_device):
    """Blocks whose expert id is -1 (not on this rank) and blocks past
    num_tokens_post_padded leave their rows untouched; fp16 activations."""
    from vllm_qdq_plugin.gemm import mxfp4_moe_linear, prepare_mxfp4_moe_weight
    m, e, top_k, bs, n, k = 24, 4, 2, 16, 256, 512
    a, codes, scales, sid, eid, ntp, topk_w = _moe_case(m, e, top_k, bs, n, k, seed=5, dtype=torch.float16)
    eid = eid.copy()
    eid[1] = -1
    sid_ext = np.concatenate([sid, np.arange(bs, dtype=np.int32)])  # a trailing block beyond ntp
    eid_ext = np.concatenate([eid, np.array([0], np.int32)])
    dev = cuda_device
    w = prepare_mxfp4_moe_weight(torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev))
    out = torch.full((m * top_k, n), 7.0, dtype=torch.float16, device=dev)
    mxfp4_moe_linear(a.to(dev), w, torch.from_numpy(sid_ext).to(dev), torch.from_numpy(eid_ext).to(dev),
                     torch.from_numpy(ntp).to(dev), None, bs, top_k, False, out=out)
    rows = og.moe_linear_exact(a.view(torch.int16).numpy().view(np.uint16), codes, scales, sid, eid,
                               int(ntp[0]), bs, top_k, fp16=True)
    got = out.float().cpu().numpy()
    skipped = [int(s) for s in sid[bs:2 * bs] if s < m * top_k]
    for s in range(m * top_k):
        if s in rows:
            _check(torch.from_numpy(got[s:s + 1]), rows[s][0][None], rows[s][1][None], f"slot {s}")
        else:
            assert s in skipped and (got[s] == 7.0).all(), s


def test_moe_marlin_hook_routes_captured_layers(cuda_device):
    """VLLM_QDQ_FUSED_GEMM=1: the patched moe_wna16_marlin_gemm runs the grouped
    FP4 GEMM for a captured MXFP4 MoE weight instead of QDQ + Marlin."""
    import os
    import types
    from unittest import mock

    from vllm_qdq_plugin import gemm, patch
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    m, e, top_k, bs, n, k = 16, 4, 2, 16, 256, 512
    a, codes, scales, sid, eid, ntp, topk_w = _moe_case(m, e, top_k, bs, n, k, seed=9)
    dev = cuda_device
    marlin_w = torch.zeros(8, dtype=torch.int32, device=dev)  # stands for the repacked expert weights
    gemm.register_marlin_moe_weight(marlin_w, gemm.prepare_mxfp4_moe_weight(
        torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev)))
    st = types.SimpleNamespace(float4_e2m1f=object(), float8_e4m3fn=object())
    ops = types.SimpleNamespace(
        moe_wna16_marlin_gemm=lambda *args: (_ for _ in ()).throw(AssertionError("Marlin called")))
    patch._patch_moe_marlin_gemm(ops, st, mxfp4_qdq, None, lambda *t: None)
    tw = torch.from_numpy(topk_w).to(dev)
    with mock.patch.dict(os.environ, {"VLLM_QDQ_FUSED_GEMM": "1"}):
        out = ops.moe_wna16_marlin_gemm(
            a.to(dev), None, marlin_w, None, torch.empty(1), None, None, None, None, None, torch.empty(1),
            torch.from_numpy(sid).to(dev), torch.from_numpy(eid).to(dev), torch.from_numpy(ntp).to(dev),
            tw, bs, top_k, True, st.float4_e2m1f, m, n, k, True, False, True, False)
    rows = og.moe_linear_exact(a.view(torch.int16).numpy().view(np.uint16), codes, scales, sid, eid,
                               int(ntp[0]), bs, top_k, topk_w.reshape(-1))
    slots = np.array(sorted(rows))
    _check(out[torch.from_numpy(slots).to(dev)], np.stack([rows[s][0] for s in slots]),
           np.stack([rows[s][1] for s in slots]), "moe hook")


@pytest.mark.parametrize("fmt", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("m,k", [(16, 2880), (40, 288), (200, 2880), (300, 288)])
def test_linear_result_independent_of_stale_workspace(cuda_device, fmt, m, k):
    """The fused linears' workspaces come from torch.empty, so they may hold
    anything an earlier tensor left, 0xFF (an E8M0 NaN) included.  With K not
    a multiple of 256 the GEMM's last K stage reads scale bytes past the
    activation's last group.  A 0x00- and a 0xFF-filled workspace must give
    the bit-identical, finite result on the decode (M <= 64) and GEMM paths."""
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.gemm import prepare_mxfp4_weight, prepare_nvfp4_weight
    dev = cuda_device
    n = 384
    a, codes, scales = _inputs(m, n, k, seed=m + k)
    ad = a.to(dev)
    lib = _native.lib()
    outs = []
    for fill in (0x00, 0xFF):
        out = torch.zeros((m, n), dtype=torch.bfloat16, device=dev)
        if fmt == "mxfp4":
            w = prepare_mxfp4_weight(torch.from_numpy(codes).to(dev), torch.from_numpy(scales).to(dev))
            ws = torch.full((lib.fp4_linear_workspace_bytes(m, k),), fill, dtype=torch.uint8, device=dev)
            _native.call("fp4_linear_mxf4", ad.data_ptr(), k, 0, w.codes.data_ptr(), w.sf_tiled.data_ptr(), 0,
                         out.data_ptr(), m, n, k, w.codes.stride(0), n, ws.data_ptr(), ws.numel(),
                         _native.stream_ptr(dev))
        else:
            # NVFP4 weight from the same nibbles with E4M3 scales per 16 in [2^-6, 2^2]
            g = torch.Generator().manual_seed(k)
            sf = (torch.randint(0x18, 0x48, (n, k // 16), generator=g)).to(torch.uint8)
            w = prepare_nvfp4_weight(torch.from_numpy(codes).to(dev), sf.to(dev), 0.5)
            ws = torch.full((lib.fp4_linear_nvf4_workspace_bytes(m, k),), fill, dtype=torch.uint8, device=dev)
            _native.call("fp4_linear_nvf4", ad.data_ptr(), k, 0, 0, w.codes.data_ptr(), w.sf_tiled.data_ptr(),
                         0.5, 0, out.data_ptr(), m, n, k, w.codes.stride(0), n, ws.data_ptr(), ws.numel(),
                         _native.stream_ptr(dev))
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.isfinite(outs[1].float()).all(), f"{fmt} m={m} k={k}: non-finite with a 0xFF workspace"
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    assert _native.device_status() == 0
