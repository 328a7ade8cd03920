"""CPU: the Marlin wrappers route activations to the QDQ hook exactly as the
reference does (reference tests/test_patch.py plus the dense-path routing of
src/vllm_qdq_plugin/patch.py:51-67)."""

from __future__ import annotations

import os
import sys
import types
from unittest import mock

import torch

from vllm_qdq_plugin import patch as P


def _scalar_types():
    return types.SimpleNamespace(float4_e2m1f=object(), float8_e4m3fn=object(),
                                 uint4b8=object())


def _moe_call(fn, x, b_q_type):
    return fn(x, None, torch.empty(1), None, torch.empty(1), None, None, None, None, None,
              torch.empty(1), torch.empty(1, dtype=torch.int32), torch.empty(1, dtype=torch.int32),
              torch.empty(1, dtype=torch.int32), torch.empty((1, 1), dtype=torch.float32),
              16, 1, False, b_q_type, 1, 1, x.shape[-1], True, False, False, False)


def _dense_call(fn, a, b_q_type):
    return fn(a, None, torch.empty(1), None, torch.empty(1), None, None, None, None, None,
              torch.empty(1), b_q_type, a.shape[0], 8, a.shape[-1])


def _raise(*a, **k):
    raise AssertionError("unexpected call")


def test_force_mxfp4_mode_applies_qdq_case_insensitively():
    st = _scalar_types()
    calls, traces = [], []
    ops = types.SimpleNamespace(moe_wna16_marlin_gemm=lambda *a, **k: a[0])

    def qdq(x, group_size=32):
        calls.append(group_size)
        return x + 1

    with mock.patch.dict(os.environ, {"VLLM_MARLIN_MOE_QDQ_MODE": "force_mxfp4"}):
        P._patch_moe_marlin_gemm(ops, st, qdq, _raise, lambda *t: traces.append(t))
        x = torch.zeros((2, 64), dtype=torch.float16)
        out = _moe_call(ops.moe_wna16_marlin_gemm, x, object())
    assert calls == [32]
    assert traces == [("moe_wna16_marlin_gemm", x.shape, x.dtype)]
    assert torch.equal(out, x + 1)


def test_force_mxfp4_mode_skips_non_2d_inputs():
    st = _scalar_types()
    calls = []
    ops = types.SimpleNamespace(moe_wna16_marlin_gemm=lambda *a, **k: a[0])
    with mock.patch.dict(os.environ, {"VLLM_MARLIN_MOE_QDQ_MODE": "FORCE_MXFP4"}):
        P._patch_moe_marlin_gemm(ops, st, lambda x, group_size=32: calls.append(group_size) or x + 1,
                                 _raise, lambda *a: None)
        x = torch.zeros((1, 2, 64), dtype=torch.float16)
        out = _moe_call(ops.moe_wna16_marlin_gemm, x, object())
    assert calls == []
    assert torch.equal(out, x)


def test_moe_routes_by_b_q_type_without_force():
    st = _scalar_types()
    seen = []
    ops = types.SimpleNamespace(moe_wna16_marlin_gemm=lambda *a, **k: a[0])
    with mock.patch.dict(os.environ, {"VLLM_MARLIN_MOE_QDQ_MODE": "0"}):
        P._patch_moe_marlin_gemm(ops, st, lambda x, group_size=32: seen.append("fp4") or x,
                                 lambda x, group_size=32: seen.append("fp8") or x,
                                 lambda *a: None)
        x = torch.zeros((3, 32), dtype=torch.bfloat16)
        _moe_call(ops.moe_wna16_marlin_gemm, x, st.float4_e2m1f)
        _moe_call(ops.moe_wna16_marlin_gemm, x, st.float8_e4m3fn)
        _moe_call(ops.moe_wna16_marlin_gemm, x, st.uint4b8)
        # no dtype check on the MoE path (reference patch.py:147)
        _moe_call(ops.moe_wna16_marlin_gemm, x.float(), st.float4_e2m1f)
    assert seen == ["fp4", "fp8", "fp4"]


def test_moe_passes_every_argument_through():
    st = _scalar_types()
    got = {}

    def orig(*args):
        got["args"] = args
        return "out"

    ops = types.SimpleNamespace(moe_wna16_marlin_gemm=orig)
    P._patch_moe_marlin_gemm(ops, st, lambda x, group_size=32: x, _raise, lambda *a: None)
    x = torch.zeros((1, 2, 64))
    assert _moe_call(ops.moe_wna16_marlin_gemm, x, object()) == "out"
    assert len(got["args"]) == 29 and got["args"][-3:] == (-1, -1, -1)


def test_dense_routing():
    st = _scalar_types()
    seen, traces = [], []
    ops = types.SimpleNamespace(marlin_gemm=lambda *a, **k: a[0])
    P._patch_marlin_gemm(ops, st, lambda x, group_size=32: seen.append(("fp4", group_size)) or x * 2,
                         lambda x, group_size=32: seen.append(("fp8", group_size)) or x * 3,
                         lambda *t: traces.append(t))
    a = torch.ones((4, 64), dtype=torch.bfloat16)
    assert torch.equal(_dense_call(ops.marlin_gemm, a, st.float4_e2m1f), a * 2)
    assert torch.equal(_dense_call(ops.marlin_gemm, a, st.float8_e4m3fn), a * 3)
    assert torch.equal(_dense_call(ops.marlin_gemm, a, st.uint4b8), a)
    # dense path checks dtype (fp16/bf16 only) and rank
    assert torch.equal(_dense_call(ops.marlin_gemm, a.float(), st.float4_e2m1f), a.float())
    a3 = torch.ones((1, 4, 64), dtype=torch.bfloat16)
    assert torch.equal(_dense_call(ops.marlin_gemm, a3, st.float4_e2m1f), a3)
    assert seen == [("fp4", 32), ("fp8", 32)]
    assert traces == [("marlin_gemm", a.shape, a.dtype)] * 2


def test_rebind_direct_imports():
    orig = object()
    new = object()
    mod = types.ModuleType("fake_consumer_mod")
    mod.marlin_gemm = orig
    sys.modules["fake_consumer_mod"] = mod
    try:
        P._rebind_direct_imports([("marlin_gemm", orig, new)])
        assert mod.marlin_gemm is new
    finally:
        del sys.modules["fake_consumer_mod"]


def test_trace_prints_first_200(capsys):
    from vllm_qdq_plugin import trace
    with mock.patch.dict(os.environ, {"VLLM_QDQ_TRACE": "1"}):
        trace._calls = 0
        for _ in range(205):
            trace.trace_qdq("marlin_gemm", (2, 3), torch.bfloat16)
    lines = capsys.readouterr().out.strip().splitlines()
    assert len(lines) == 200
    assert lines[0] == "[QDQ] op=marlin_gemm shape=(2, 3) dtype=torch.bfloat16"
    trace._calls = 0


def test_register_is_gated_on_vllm_qdq():
    import vllm_qdq_plugin
    with mock.patch.dict(os.environ, {"VLLM_QDQ": "0"}), \
            mock.patch.object(P, "apply_patches", side_effect=_raise):
        vllm_qdq_plugin.register()
    called = []
    with mock.patch.dict(os.environ, {"VLLM_QDQ": "1"}), \
            mock.patch.object(P, "apply_patches", side_effect=lambda: called.append(1)):
        vllm_qdq_plugin.register()
    assert called == [1]


def test_nvfp4_activation_knob_on_nvfp4_layers():
    """VLLM_QDQ_NVFP4_ACT=1 (this build only): float4_e2m1f layers that carry a
    global scale (vLLM's NVFP4 Marlin layers) get NVFP4 QDQ; MXFP4 layers and
    the knob's default keep the reference's MXFP4 QDQ."""
    st = _scalar_types()
    seen = []
    ops = types.SimpleNamespace(marlin_gemm=lambda *a, **k: a[0],
                                moe_wna16_marlin_gemm=lambda *a, **k: a[0])

    def fake_nv(x, group_size=16, global_scale=None):
        seen.append(("nv", group_size))
        return x * 5

    def mx(x, group_size=32):
        seen.append(("mx", group_size))
        return x * 2

    gs = torch.ones(1)
    a = torch.ones((4, 64), dtype=torch.bfloat16)

    def dense(global_scale):
        return ops.marlin_gemm(a, None, torch.empty(1), None, torch.empty(1), None, global_scale, None,
                               None, None, torch.empty(1), st.float4_e2m1f, 4, 8, 64)

    def moe(global_scale):
        return ops.moe_wna16_marlin_gemm(
            a, None, torch.empty(1), None, torch.empty(1), None, global_scale, None, None, None,
            torch.empty(1), torch.empty(1, dtype=torch.int32), torch.empty(1, dtype=torch.int32),
            torch.empty(1, dtype=torch.int32), torch.empty((1, 1)), 16, 1, False, st.float4_e2m1f,
            4, 8, 64, True, False, False, False)

    P._patch_marlin_gemm(ops, st, mx, _raise, lambda *t: None)
    P._patch_moe_marlin_gemm(ops, st, mx, _raise, lambda *t: None)
    with mock.patch("vllm_qdq_plugin.qdq.nvfp4.nvfp4_qdq", fake_nv):
        with mock.patch.dict(os.environ, {"VLLM_QDQ_NVFP4_ACT": "1", "VLLM_MARLIN_MOE_QDQ_MODE": "0"}):
            assert torch.equal(dense(gs), a * 5)
            assert torch.equal(dense(None), a * 2)
            assert torch.equal(moe(gs), a * 5)
            assert torch.equal(moe(None), a * 2)
        with mock.patch.dict(os.environ, {"VLLM_QDQ_NVFP4_ACT": "0", "VLLM_MARLIN_MOE_QDQ_MODE": "0"}):
            assert torch.equal(dense(gs), a * 2)
            assert torch.equal(moe(gs), a * 2)
        with mock.patch.dict(os.environ, {"VLLM_QDQ_NVFP4_ACT": "1",
                                          "VLLM_MARLIN_MOE_QDQ_MODE": "FORCE_MXFP4"}):
            assert torch.equal(moe(gs), a * 2)  # FORCE_MXFP4 keeps precedence, as in the reference
    assert seen == [("nv", 16), ("mx", 32), ("nv", 16), ("mx", 32), ("mx", 32), ("mx", 32), ("mx", 32)]
