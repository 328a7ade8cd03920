"""CPU: per-(layer, denoising-step) routing of the Sage3 config
(reference behaviour: tests/test_route_table.py, tests/test_patch_attention.py
of the plugin; src/vllm_qdq_plugin/sage3_attn/routing/*).  vllm-omni is not
installed here, so its attention module is a stub class."""

from __future__ import annotations

import json
import sys
import types
from unittest import mock

import pytest
import torch

from vllm_qdq_plugin.sage3_attn.impl import Sage3TritonImpl
from vllm_qdq_plugin.sage3_attn.routing import patch_attention as P
from vllm_qdq_plugin.sage3_attn.routing.route_table import IntervalSet, RouteTable, route_vocabulary


def _route(tmp_path, data, name="route.json") -> str:
    path = tmp_path / name
    path.write_text(json.dumps(data))
    return str(path)


# ------------------------------------------------------------------ ranges
@pytest.mark.parametrize("spec,want", [
    ("0-7,9,12-15", set(range(8)) | {9} | set(range(12, 16))),
    ("5", {5}), ("3-3", {3}), ("", set()), (" 1 - 3 , 5 ", {1, 2, 3, 5}),
])
def test_parse_ranges(spec, want):
    assert IntervalSet.parse(spec) == want
    assert all(x in IntervalSet.parse(spec) for x in want)
    assert -1 not in IntervalSet.parse(spec) and 10**6 not in IntervalSet.parse(spec)


def test_intervals_are_sorted_and_merged():
    assert IntervalSet.parse("12-15,0-3,4-7,9,6-8").intervals() == [(0, 9), (12, 15)]
    assert IntervalSet.parse(7).intervals() == [(7, 7)]
    assert None not in IntervalSet.parse("0-3")


@pytest.mark.parametrize("spec", ["7-3", "a-b", "1-x", "-2", "1-2-3"])
def test_parse_ranges_rejects(spec):
    with pytest.raises(ValueError):
        IntervalSet.parse(spec)


# ------------------------------------------------------------------ resolution
@pytest.fixture
def table(tmp_path):
    return RouteTable.from_json_file(_route(tmp_path, {
        "default": "mxfp4",
        "rules": [{"layers": "20-39", "steps": "0-7", "config": "mixed_fp8qk_fp4pv"},
                  {"steps": "0-7", "config": "sdpa"},
                  {"layers": "20-39", "config": "mxfp8_s1"}]}))


@pytest.mark.parametrize("layer,step,want", [
    (25, 3, "mixed_fp8qk_fp4pv"),   # first rule wins when both predicates match
    (5, 3, "sdpa"),                 # step-only rule
    (25, 50, "mxfp8_s1"),           # layer-only rule
    (5, 50, "mxfp4"),               # default
    (None, 3, "sdpa"),              # unknown layer cannot satisfy a layer predicate
    (25, None, "mxfp8_s1"),
    (None, None, "mxfp4"),
])
def test_resolve(table, layer, step, want):
    assert table.resolve(layer, step) == want


def test_load_rules(tmp_path):
    t = RouteTable.from_json_file(_route(tmp_path, {"rules": [{"layers": "0-5", "config": "mxfp4"}]}))
    assert t.resolve(99, 0) is None and t.resolve(3, 0) == "mxfp4"
    t = RouteTable.from_json_file(_route(tmp_path, {"rules": [{"layers": 7, "steps": 0, "config": "mxfp4"}]}))
    assert t.resolve(7, 0) == "mxfp4" and t.resolve(8, 0) is None
    assert RouteTable.from_json_file(_route(tmp_path, {"default": "sdpa", "rules": []})).resolve(0, 0) == "sdpa"
    # every config name the reference registers is a valid route target
    assert {"mxfp4_s1_e4m3", "mixed_fp4qk_fp8pv_vs", "mxfp8_hw", "sdpa"} <= route_vocabulary()


@pytest.mark.parametrize("data", [
    {"rules": [{"config": "not_a_real_config"}]},
    {"default": "nope", "rules": []},
    {"rules": [{"layers": "0-5"}]},
    [],
    {"rules": {}},
    {"rules": ["mxfp4"]},
    {"rules": [{"layers": True, "config": "mxfp4"}]},
    {"rules": [{"layers": 1.5, "config": "mxfp4"}]},
])
def test_load_rejects(tmp_path, data):
    with pytest.raises(ValueError):
        RouteTable.from_json_file(_route(tmp_path, data))


# ------------------------------------------------------------------ dispatch
@pytest.fixture
def routed(tmp_path):
    saved = (P._installed, P._ORIG, P._TABLE)
    P._TABLE = RouteTable.from_json_file(_route(tmp_path, {
        "default": "mxfp4", "rules": [{"steps": "0-3", "config": "sdpa"},
                                      {"layers": "20-39", "config": "mxfp8_s1"}]}))
    P._ORIG = lambda self, q, k, v, m: "ORIG"
    yield
    P._installed, P._ORIG, P._TABLE = saved


def _impl():
    impl = mock.MagicMock(spec=Sage3TritonImpl)
    impl.forward_cuda.return_value = "CUDA"
    impl._forward_sdpa.return_value = "SDPA"
    return impl


def _module(role="self", layer_idx=0, impl=None):
    return types.SimpleNamespace(role=role, layer_idx=layer_idx, attention=impl if impl is not None else _impl())


def _run(module, dtype=torch.bfloat16, step=None, ctx=True):
    q = torch.zeros(1, 4, 2, 8, dtype=dtype)
    with mock.patch.object(P, "is_forward_context_available", return_value=ctx), \
            mock.patch.object(P, "get_forward_context", return_value=types.SimpleNamespace(denoise_step_idx=step)):
        return P._routed_run_local_attention(module, q, q, q, None)


def test_dispatch_falls_through(routed):
    assert _run(_module(), dtype=torch.float32) == "ORIG"
    assert _run(_module(role="cross")) == "ORIG"
    assert _run(types.SimpleNamespace(role="self", layer_idx=0, attention=object())) == "ORIG"


def test_dispatch_routes(routed):
    impl = _impl()
    assert _run(_module(layer_idx=25, impl=impl), step=2) == "SDPA"
    impl._forward_sdpa.assert_called_once()
    impl.forward_cuda.assert_not_called()
    impl = _impl()
    assert _run(_module(layer_idx=25, impl=impl), step=50) == "CUDA"
    assert impl.forward_cuda.call_args.kwargs["config_override"] == "mxfp8_s1"
    impl = _impl()
    _run(_module(layer_idx=5, impl=impl), step=50)
    assert impl.forward_cuda.call_args.kwargs["config_override"] == "mxfp4"
    impl = _impl()   # no forward context: the step is unknown
    _run(_module(layer_idx=25, impl=impl), ctx=False)
    assert impl.forward_cuda.call_args.kwargs["config_override"] == "mxfp8_s1"


def test_dispatch_without_match_calls_original(routed, tmp_path):
    P._TABLE = RouteTable.from_json_file(_route(tmp_path, {"rules": [{"layers": "20-39", "config": "mxfp4"}]},
                                                "r2.json"))
    impl = _impl()
    assert _run(_module(layer_idx=5, impl=impl), step=0) == "ORIG"
    impl.forward_cuda.assert_not_called()


# ------------------------------------------------------------------ install
@pytest.fixture
def fake_omni(monkeypatch):
    class Attention:
        def _run_local_attention(self, q, k, v, m):
            return "ORIG"

    names = ["vllm_omni", "vllm_omni.diffusion", "vllm_omni.diffusion.attention",
             "vllm_omni.diffusion.attention.layer"]
    for n in names:
        monkeypatch.setitem(sys.modules, n, types.ModuleType(n))
    sys.modules["vllm_omni.diffusion.attention.layer"].Attention = Attention
    saved = (P._installed, P._ORIG, P._TABLE)
    P._installed, P._ORIG, P._TABLE = False, None, None
    yield Attention
    P._installed, P._ORIG, P._TABLE = saved


def test_install_is_idempotent(fake_omni, tmp_path):
    path = _route(tmp_path, {"default": "mxfp4", "rules": [{"steps": "0-3", "config": "sdpa"}]})
    original = fake_omni._run_local_attention
    P.install(path)
    assert fake_omni._run_local_attention is P._routed_run_local_attention
    assert P._ORIG is original and P._installed and P._TABLE.default == "mxfp4"
    P.install(path)
    assert P._ORIG is original


def test_install_rejects_bad_file_without_patching(fake_omni, tmp_path):
    original = fake_omni._run_local_attention
    with pytest.raises(ValueError):
        P.install(_route(tmp_path, {"rules": [{"config": "not_real"}]}))
    assert not P._installed and fake_omni._run_local_attention is original


def test_register_omni_survives_a_bad_route_file(tmp_path, monkeypatch):
    import vllm_qdq_plugin as plugin
    saved = (P._installed, P._ORIG, P._TABLE)
    P._installed = False
    try:
        plugin._maybe_install_route(_route(tmp_path, {"rules": [{"config": "not_real"}]}))
        assert not P._installed
        plugin._maybe_install_route("")
    finally:
        P._installed, P._ORIG, P._TABLE = saved
