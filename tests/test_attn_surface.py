"""CPU: the SAGE_ATTN backend surface for calls the FP4 kernels do not take.

The backend advertises the reference's head sizes, 32-256
(src/vllm_qdq_plugin/sage3_attn/backend.py:18-20); the FP4 kernels take 32,
64, 96 and 128 with bf16 or fp16 inputs.  A head dim or dtype outside that runs SDPA
with a warning instead of failing in forward; the acc_dtype knob is validated and a non-fp32 mode is logged once.
"""

from __future__ import annotations

import logging

import pytest
import torch
import torch.nn.functional as F

from vllm_qdq_plugin.sage3_attn import impl as impl_mod
from vllm_qdq_plugin.sage3_attn.backend import Sage3TritonBackend
from vllm_qdq_plugin.sage3_attn.impl import Sage3TritonImpl
from vllm_qdq_plugin.sage3_attn.sage3 import api


def _sdpa_nhd(q, k, v, scale):
    return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                          scale=scale).transpose(1, 2)


@pytest.mark.parametrize("d,dtype", [(256, torch.bfloat16), (160, torch.bfloat16), (224, torch.float16),
                                     (128, torch.float32), (64, torch.float32)])
def test_unsupported_head_dim_or_dtype_runs_sdpa(d, dtype, caplog):
    assert d in Sage3TritonBackend.get_supported_head_sizes() or dtype == torch.float32
    g = torch.Generator().manual_seed(d)
    q, k, v = (torch.randn(1, 40, 2, d, generator=g).to(dtype) for _ in range(3))
    impl = Sage3TritonImpl(num_heads=2, head_size=d, softmax_scale=d ** -0.5)
    impl_mod._WARNED.clear()
    with caplog.at_level(logging.WARNING):
        out = impl.forward_cuda(q, k, v)
        impl.forward_cuda(q, k, v)
    assert out.shape == q.shape and out.dtype == dtype
    torch.testing.assert_close(out, _sdpa_nhd(q, k, v, d ** -0.5))
    assert sum("runs SDPA instead" in r.getMessage() for r in caplog.records) == 1


def test_supported_shape_is_not_rerouted():
    for d in (32, 64, 96, 128):
        for dtype in (torch.bfloat16, torch.float16):
            assert api.unsupported_reason(torch.zeros(1, 8, 2, d, dtype=dtype)) is None
    assert "head_dim 256" in api.unsupported_reason(torch.zeros(1, 8, 2, 256, dtype=torch.bfloat16))
    assert "float32" in api.unsupported_reason(torch.zeros(1, 8, 2, 128, dtype=torch.float32))


def test_acc_dtype_validated_and_logged_once(caplog):
    with pytest.raises(ValueError):
        api._acc_mode("fp8_everything")
    api._ACC_WARNED.clear()
    with caplog.at_level(logging.WARNING):
        assert api._acc_mode("fp32") == 0
        assert api._acc_mode("bf16_pv_only") == 1
        assert api._acc_mode("bf16_pv_only") == 1
    msgs = [r.getMessage() for r in caplog.records if "SAGE3_ACC_DTYPE" in r.getMessage()]
    assert len(msgs) == 1 and "bf16_pv_only" in msgs[0]
