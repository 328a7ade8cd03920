"""GPU parity of the sm_100a Sage3 FP4 / FP8 attention (through the C ABI).

Oracle: oracle/attn.py, a numpy restatement of the reference's paths
(qk_smoothing + FP4 quantisation + the flash loop).  The kernel steps its
online softmax over 128-key tiles for every config; the tight comparison
runs the oracle with the same tile (KERNEL_BLOCK_N).  The reference's own
tiles are 64 keys for mxfp4_hw (mxfp4_hw_kernel.py:437) and 128 for the
emulated mxfp4 / nvfp4 configs (attention_kernel.py:249-253), the oracle's
defaults, which the accuracy comparison uses.  Tolerances (floating point):
relative L2 error vs the same-tile oracle <= 2e-2 (the kernel's exp2 is the
hardware approximation, so a few P codes sit on the other side of a rounding
boundary), and the quantisation error vs exact float64 attention within 1.1x
(+0.01) of the reference-tiled oracle's error vs exact attention.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attn as oa

pytestmark = pytest.mark.gpu

KERNEL_BLOCK_N = 128  # keys per online-softmax step of the flash kernel


def _qkv(L, H, seed, k_offset=3.0, B=1, v_offset=0.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, L, H, 128, generator=g)
    k = torch.randn(B, L, H, 128, generator=g) + torch.randn(B, 1, H, 128, generator=g) * k_offset
    v = torch.randn(B, L, H, 128, generator=g)
    if v_offset:
        v = v + torch.randn(B, 1, H, 128, generator=g) * v_offset
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _run(q, k, v, dev, causal=False, config="mxfp4_hw", smoothing=True):
    from vllm_qdq_plugin.sage3_attn.sage3 import sage3_attention_nhd
    out = sage3_attention_nhd(q.to(dev), k.to(dev), v.to(dev), config=config, is_causal=causal,
                              per_block_mean=smoothing)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("L,H", [(128, 1), (256, 2), (300, 2), (1000, 1)])
def test_mxfp4_attention_matches_oracle(cuda_device, L, H):
    q, k, v = _qkv(L, H, seed=L + H)
    sm = 1.0 / math.sqrt(128)
    got = _run(q, k, v, cuda_device)[0]
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N)
    err = oa.rel_l2(got, want)
    assert err < 2e-2, f"rel L2 vs oracle {err}"
    exact = oa.exact_attention(qb, kb, vb, sm)
    ref_err = oa.rel_l2(oa.attention(qb, kb, vb, sm, mask_padding=False), exact)
    our_err = oa.rel_l2(got, exact)
    assert our_err <= 1.1 * ref_err + 0.01, (our_err, ref_err)
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


@pytest.mark.parametrize("config", ["mxfp4", "nvfp4"])
@pytest.mark.parametrize("L,H", [(256, 2), (1000, 1)])
def test_emulated_configs_match_oracle(cuda_device, config, L, H):
    q, k, v = _qkv(L, H, seed=L * 3 + H)
    sm = 1.0 / math.sqrt(128)
    got = _run(q, k, v, cuda_device, config=config)[0]
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, config=config)
    assert oa.rel_l2(got, want) < 2e-2, oa.rel_l2(got, want)
    exact = oa.exact_attention(qb, kb, vb, sm)
    assert oa.rel_l2(got, exact) <= 1.1 * oa.rel_l2(want, exact) + 0.01


@pytest.mark.parametrize("config", ["mxfp4_hw", "nvfp4", "mxfp8_hw", "mxfp4_s1_vsmooth"])
@pytest.mark.parametrize("L,H,causal", [(300, 2, False), (1000, 1, False), (256, 1, True)])
def test_fp16_inputs_match_oracle(cuda_device, config, L, H, causal):
    """fp16 q/k/v: the smoothing rounds to fp16 (as the reference's torch ops
    on fp16 tensors), delta_s is an fp16 MMA operand and the output is fp16.
    Same bars as bf16: relative L2 vs the same-tile oracle (run with fp16
    roundings) <= 2e-2, error vs exact attention within 1.1x (+0.01) of the
    reference-tiled oracle's."""
    q, k, v = (t.to(torch.float16) for t in _qkv(L, H, seed=L * 5 + H + len(config), v_offset=2.0))
    sm = 1.0 / math.sqrt(128)
    from vllm_qdq_plugin.sage3_attn.sage3 import sage3_attention_nhd
    out = sage3_attention_nhd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), config=config,
                              is_causal=causal)
    assert out.dtype == torch.float16
    got = out.float().cpu().numpy()[0]
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, causal=causal, config=config, f16=True)
    err = oa.rel_l2(got, want)
    assert err < 2e-2, f"rel L2 vs oracle {err}"
    exact = oa.exact_attention(qb, kb, vb, sm, causal=causal, f16=True)
    ref = oa.attention(qb, kb, vb, sm, causal=causal, config=config, mask_padding=False, f16=True)
    assert oa.rel_l2(got, exact) <= 1.1 * oa.rel_l2(ref, exact) + 0.01
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


SINGLE_LEVEL_AND_MIXED = ["mxfp4_s1", "mxfp8_s1", "mixed_fp8qk_fp4pv", "mixed_fp4qk_fp8pv",
                          "mixed_mxfp8qk_mxfp4pv_hw", "mixed_mxfp4qk_mxfp8pv_hw", "mxfp4_s1_vsmooth",
                          "mixed_fp8qk_fp4pv_vs", "mixed_fp4qk_fp8pv_vs", "mxfp4_s1_2level", "mxfp4_s1_e4m3"]


@pytest.mark.parametrize("config", SINGLE_LEVEL_AND_MIXED)
@pytest.mark.parametrize("L,H,causal", [(256, 2, False), (1000, 1, False), (300, 1, True)])
def test_single_level_and_mixed_configs_match_oracle(cuda_device, config, L, H, causal):
    """Single-level (_s1), mixed-format and V-smoothed configs: relative L2 vs
    the same-tile oracle <= 2e-2 and the error vs exact attention within 1.1x
    (+0.01) of the oracle's.  V carries a per-channel offset so that V
    smoothing changes the quantised operand."""
    q, k, v = _qkv(L, H, seed=L * 7 + H + len(config), v_offset=2.0)
    sm = 1.0 / math.sqrt(128)
    got = _run(q, k, v, cuda_device, causal=causal, config=config)[0]
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, causal=causal, config=config)
    err = oa.rel_l2(got, want)
    assert err < 2e-2, f"rel L2 vs oracle {err}"
    exact = oa.exact_attention(qb, kb, vb, sm, causal=causal)
    assert oa.rel_l2(got, exact) <= 1.1 * oa.rel_l2(want, exact) + 0.01
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


def test_v_smoothing_reduces_error(cuda_device):
    """With a large per-channel V offset, subtracting the V mean before the FP4
    quantisation (mxfp4_s1_vsmooth) gives a smaller error than mxfp4_s1."""
    q, k, v = _qkv(512, 2, seed=31, v_offset=8.0)
    sm = 1.0 / math.sqrt(128)
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    exact = oa.exact_attention(qb, kb, vb, sm)
    plain = oa.rel_l2(_run(q, k, v, cuda_device, config="mxfp4_s1")[0], exact)
    smooth = oa.rel_l2(_run(q, k, v, cuda_device, config="mxfp4_s1_vsmooth")[0], exact)
    assert smooth < 0.8 * plain, (smooth, plain)


@pytest.mark.parametrize("config", ["mixed_fp8qk_fp4pv", "mixed_mxfp4qk_mxfp8pv_hw", "mxfp4_s1_vsmooth",
                                    "mxfp4_s1_e4m3", "mxfp4", "mxfp8_s1"])
def test_new_config_prepass_codes_bit_exact(cuda_device, config):
    """The pre-pass codes and scales of q_s, k_c and V (mean-subtracted for the
    V-smoothed configs), read back from the workspace, dequantise to exactly
    the oracle's values in each operand format; for the emulated E8M0 configs
    (mxfp4, mxfp8_s1, the mixed and V-smoothed ones) those are the
    reference's own quantize_qk / quantize_v values (9-level grid or E4M3,
    scale arithmetic in bf16)."""
    import ctypes
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.sage3_attn.sage3 import api
    qk_fmt, pv_fmt, _, _, vsmooth, qk_smooth = oa.CONFIGS[config]
    L, H = 300, 1
    q, k, v = _qkv(L, H, seed=29, v_offset=2.0)
    dev = cuda_device
    qd_, kd_, vd_ = (t.to(dev) for t in (q, k, v))
    out = torch.empty_like(qd_)
    lib = _native.lib()
    nbytes = lib.sage3_attn_workspace_bytes(1, L, H, 128)
    ws = torch.zeros((nbytes,), dtype=torch.uint8, device=dev)
    st = [qd_.stride(0), qd_.stride(1), qd_.stride(2)] * 3 + [out.stride(0), out.stride(1), out.stride(2)]
    _native.call("sage3_fp4_attn", qd_.data_ptr(), kd_.data_ptr(), vd_.data_ptr(), out.data_ptr(), 1, L, H, 128,
                 (ctypes.c_int64 * 12)(*st), 1.0 / math.sqrt(128), api.ATTENTION_CONFIGS[config], 0, 0,
                 api._smoothing_flags(config, True), 0, ws.data_ptr(), nbytes, _native.stream_ptr(dev))
    torch.cuda.synchronize()
    w = ws.cpu().numpy()
    Lp, G = 384, 3
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    e4m3 = ("mx8", "g9", "e8")  # formats held as E4M3 codes (the 9-level grid values are E4M3 values)
    row = lambda fmt: 128 if fmt in e4m3 else 64  # noqa: E731

    def deq(fmt, c, sc):
        if fmt in e4m3:
            return oa._deq8(c, sc)
        if fmt == "nv4b32":  # E2M1 codes, E4M3 scale bytes per 32
            vals = np.stack([oa.E2M1[c & 0xF], oa.E2M1[c >> 4]], axis=-1).reshape(c.shape[0], -1)
            return vals * np.repeat(oa.E4M3[sc], 32, axis=-1)
        return oa._deq(c, sc)

    def sf(buf):
        if qk_fmt != "nv4b32" and pv_fmt != "nv4b32":
            return _sf_tile(buf, G)
        # 8 slots of 16 per row in two chunks; each per-32 scale fills two adjacent slots
        both = np.concatenate([_sf_tile(buf, G), _sf_tile(buf[512:], G)], axis=1)
        np.testing.assert_array_equal(both[:, 0::2], both[:, 1::2])
        return both[:, 0::2]

    off = up(128 * 4) + up(G * 128 * 2)
    qc = w[off: off + Lp * row(qk_fmt)].reshape(Lp, row(qk_fmt)); off += up(Lp * 128)
    qsf = sf(w[off:]); off += up(G * 1024)
    kc = w[off: off + Lp * row(qk_fmt)].reshape(Lp, row(qk_fmt)); off += up(Lp * 128)
    ksf = sf(w[off:]); off += up(G * 1024)
    vrow = Lp if pv_fmt in e4m3 else Lp // 2
    vt = w[off: off + 128 * vrow].reshape(128, vrow); off += up(128 * Lp)
    vsf = sf(w[off:]).reshape(G, 128, 4).transpose(1, 0, 2).reshape(128, G * 4)
    f = lambda t: oa.bf16_bits_to_f32(_bits(t[0, :, 0]))  # noqa: E731
    qd, kd, vd, _ = oa.prepass(f(q), f(k), f(v), qk_smooth, qk_fmt=qk_fmt, pv_fmt=pv_fmt, vsmooth=vsmooth)
    np.testing.assert_array_equal(deq(qk_fmt, qc, qsf), qd)
    np.testing.assert_array_equal(deq(qk_fmt, kc, ksf), kd)
    np.testing.assert_array_equal(deq(pv_fmt, vt, vsf).T, vd)


def test_config5_flux_shape_nvfp4(cuda_device):
    """BASELINE config 5 distribution (1% of K rows x20) on a reduced batch."""
    g = torch.Generator().manual_seed(5)
    B, L, H = 1, 512, 2
    q = torch.randn(B, L, H, 128, generator=g)
    k = torch.randn(B, L, H, 128, generator=g)
    rows = torch.randperm(L, generator=g)[: L // 100]
    k[:, rows] *= 20
    v = torch.randn(B, L, H, 128, generator=g)
    q, k, v = (t.to(torch.bfloat16) for t in (q, k, v))
    from vllm_qdq_plugin.sage3_attn.sage3 import sage3_attention_nhd
    got = sage3_attention_nhd(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), config="nvfp4",
                              acc_dtype="bf16_pv_only").float().cpu().numpy()[0]
    sm = 1.0 / math.sqrt(128)
    want = oa.attention(_bits(q[0]), _bits(k[0]), _bits(v[0]), sm, block_n=KERNEL_BLOCK_N, config="nvfp4")
    assert oa.rel_l2(got, want) < 2e-2


@pytest.mark.parametrize("L,H", [(128, 1), (300, 2), (1000, 1)])
def test_mxfp8_attention_matches_oracle(cuda_device, L, H):
    """mxfp8_hw (E4M3 Q/K/V/P on kind::mxf8f6f4): relative L2 vs the same-tile
    oracle <= 1e-2, and the error vs exact attention within 1.1x (+0.005) of
    the reference-tiled oracle's."""
    q, k, v = _qkv(L, H, seed=L + 5 * H)
    sm = 1.0 / math.sqrt(128)
    got = _run(q, k, v, cuda_device, config="mxfp8_hw")[0]
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, config="mxfp8_hw")
    err = oa.rel_l2(got, want)
    assert err < 1e-2, f"rel L2 vs oracle {err}"
    exact = oa.exact_attention(qb, kb, vb, sm)
    ref_err = oa.rel_l2(oa.attention(qb, kb, vb, sm, mask_padding=False, config="mxfp8_hw"), exact)
    our_err = oa.rel_l2(got, exact)
    assert our_err <= 1.1 * ref_err + 0.005, (our_err, ref_err)
    # MXFP8 is far closer to exact attention than MXFP4
    assert our_err < 0.5 * oa.rel_l2(oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N), exact)
    from vllm_qdq_plugin import _native
    assert _native.device_status() == 0


def test_mxfp8_causal_and_no_smoothing(cuda_device):
    q, k, v = _qkv(384, 1, seed=17)
    sm = 1.0 / math.sqrt(128)
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    got = _run(q, k, v, cuda_device, causal=True, config="mxfp8_hw")[0]
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, causal=True, config="mxfp8_hw")
    assert oa.rel_l2(got, want) < 1e-2
    got = _run(q, k, v, cuda_device, smoothing=False, config="mxfp8_hw")[0]
    want = oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, smoothing=False, config="mxfp8_hw")
    assert oa.rel_l2(got, want) < 1e-2


def _sf_tile(buf: np.ndarray, tiles: int) -> np.ndarray:
    """Scale bytes [tiles * 128, 4] from 1024-byte tcgen05 chunks (row r, group g
    at (r % 32) * 16 + (r // 32) * 4 + g of the first 512 bytes)."""
    t = buf[: tiles * 1024].reshape(tiles, 1024)[:, :512].reshape(tiles, 32, 4, 4)  # [tile, r%32, r//32, g]
    return t.transpose(0, 2, 1, 3).reshape(tiles * 128, 4)


def test_mxfp8_prepass_codes_bit_exact(cuda_device):
    """The pre-pass's E4M3 codes and E8M0 scales of q_s, k_c (along D) and V
    (along the sequence), read back from the workspace, dequantise to exactly
    the oracle's quantize_to_mxfp8 values (smoothing included)."""
    import ctypes
    from vllm_qdq_plugin import _native
    L, H = 300, 1
    q, k, v = _qkv(L, H, seed=23)
    dev = cuda_device
    qd_, kd_, vd_ = (t.to(dev) for t in (q, k, v))
    out = torch.empty_like(qd_)
    lib = _native.lib()
    nbytes = lib.sage3_attn_workspace_bytes(1, L, H, 128)
    ws = torch.zeros((nbytes,), dtype=torch.uint8, device=dev)
    st = [qd_.stride(0), qd_.stride(1), qd_.stride(2)] * 3 + [out.stride(0), out.stride(1), out.stride(2)]
    _native.call("sage3_fp4_attn", qd_.data_ptr(), kd_.data_ptr(), vd_.data_ptr(), out.data_ptr(), 1, L, H, 128,
                 (ctypes.c_int64 * 12)(*st), 1.0 / math.sqrt(128), 3, 0, 0, 1, 0, ws.data_ptr(), nbytes,
                 _native.stream_ptr(dev))
    torch.cuda.synchronize()
    w = ws.cpu().numpy()
    Lp, G = 384, 3
    up = lambda n: (n + 255) // 256 * 256  # noqa: E731
    off = up(128 * 4) + up(G * 128 * 2)
    qc = w[off: off + Lp * 128].reshape(Lp, 128); off += up(Lp * 128)
    qsf = _sf_tile(w[off:], G); off += up(G * 1024)
    kc = w[off: off + Lp * 128].reshape(Lp, 128); off += up(Lp * 128)
    ksf = _sf_tile(w[off:], G); off += up(G * 1024)
    vt = w[off: off + 128 * Lp].reshape(128, Lp); off += up(128 * Lp)
    vsf = _sf_tile(w[off:], G).reshape(G, 128, 4).transpose(1, 0, 2).reshape(128, G * 4)  # [d, key group]
    qd, kd, vd, _ = oa.prepass(oa.bf16_bits_to_f32(_bits(q[0, :, 0])), oa.bf16_bits_to_f32(_bits(k[0, :, 0])),
                               oa.bf16_bits_to_f32(_bits(v[0, :, 0])), True, False, True)
    np.testing.assert_array_equal(oa._deq8(qc, qsf), qd)
    np.testing.assert_array_equal(oa._deq8(kc, ksf), kd)
    np.testing.assert_array_equal(oa._deq8(vt, vsf).T, vd)


def test_causal_and_no_smoothing(cuda_device):
    q, k, v = _qkv(384, 1, seed=7)
    sm = 1.0 / math.sqrt(128)
    qb, kb, vb = _bits(q[0]), _bits(k[0]), _bits(v[0])
    got = _run(q, k, v, cuda_device, causal=True)[0]
    assert oa.rel_l2(got, oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, causal=True)) < 2e-2
    got = _run(q, k, v, cuda_device, smoothing=False)[0]
    assert oa.rel_l2(got, oa.attention(qb, kb, vb, sm, block_n=KERNEL_BLOCK_N, smoothing=False)) < 2e-2


def test_batch_heads_and_hnd_layout(cuda_device):
    from vllm_qdq_plugin.sage3_attn.sage3 import sageattn3_standalone
    q, k, v = _qkv(256, 3, seed=11, B=2)
    nhd = _run(q, k, v, cuda_device)
    hnd = sageattn3_standalone(q.transpose(1, 2).to(cuda_device), k.transpose(1, 2).to(cuda_device),
                               v.transpose(1, 2).to(cuda_device), config="mxfp4_hw")
    assert np.array_equal(hnd.transpose(1, 2).float().cpu().numpy(), nhd)
    sm = 1.0 / math.sqrt(128)
    for b in range(2):
        want = oa.attention(_bits(q[b]), _bits(k[b]), _bits(v[b]), sm, block_n=KERNEL_BLOCK_N)
        assert oa.rel_l2(nhd[b], want) < 2e-2


def test_backend_impl_surface(cuda_device):
    from vllm_qdq_plugin.sage3_attn.backend import Sage3TritonBackend
    impl_cls = Sage3TritonBackend.get_impl_cls()
    impl = impl_cls(num_heads=2, head_size=128, softmax_scale=1 / math.sqrt(128),
                    backend_kwargs={"sage3_config": "mxfp4_hw"})
    q, k, v = _qkv(200, 2, seed=5)
    out = impl.forward_cuda(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    assert out.shape == q.shape and out.dtype == torch.bfloat16
    # cross-attention falls back to SDPA
    kv = _qkv(64, 2, seed=6)
    out2 = impl.forward_cuda(q.to(cuda_device), kv[1].to(cuda_device), kv[2].to(cuda_device))
    assert out2.shape == q.shape
