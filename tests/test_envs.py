"""CPU: the lazy env module keeps the reference's names, defaults and validation
(reference tests/test_envs.py)."""

from __future__ import annotations

import os
from unittest import mock

import pytest

from vllm_qdq_plugin import envs


def test_case_insensitive_choice_returns_canonical_value():
    with mock.patch.dict(os.environ, {"VLLM_MARLIN_MOE_QDQ_MODE": "force_mxfp4"}):
        assert envs.VLLM_MARLIN_MOE_QDQ_MODE == "FORCE_MXFP4"


def test_invalid_choice_raises():
    with mock.patch.dict(os.environ, {"VLLM_MARLIN_MOE_QDQ_MODE": "bad_mode"}):
        with pytest.raises(ValueError, match="Invalid value 'bad_mode'"):
            _ = envs.VLLM_MARLIN_MOE_QDQ_MODE


def test_defaults_and_flags():
    keys = ["SAGE3_QUANT_FORMAT", "SAGE3_ACC_DTYPE", "VLLM_QDQ", "VLLM_QDQ_TRACE",
            "VLLM_MARLIN_MOE_QDQ_MODE", "VLLM_SAGE3_TRITON"]
    clean = {k: v for k, v in os.environ.items() if k not in keys}
    with mock.patch.dict(os.environ, clean, clear=True):
        assert envs.SAGE3_QUANT_FORMAT == "mxfp4"
        assert envs.SAGE3_ACC_DTYPE == "fp32"
        assert envs.VLLM_QDQ is False
        assert envs.VLLM_MARLIN_MOE_QDQ_MODE == "0"
        assert not envs.is_set("VLLM_QDQ")
    for val, expect in (("1", True), ("TRUE", True), ("yes", True), ("0", False), ("no", False)):
        with mock.patch.dict(os.environ, {"VLLM_QDQ": val}):
            assert envs.VLLM_QDQ is expect
            assert envs.is_set("VLLM_QDQ")


def test_unknown_attribute():
    with pytest.raises(AttributeError):
        _ = envs.NOT_A_KNOB
    assert "VLLM_QDQ" in dir(envs)
