"""Failure detection without a GPU fault.

A kernel waits on an mbarrier that nothing arrives at; its bounded wait must
give up after a short limit, record QDQ_ERR_TIMEOUT in the device status word
(read on the host through qdq_device_status) and exit, leaving the CUDA
context usable for the next kernels.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT = 4
SITE = 0x7E57


def test_bounded_wait_times_out_and_context_survives(cuda_device):
    from oracle import qdq as oq
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.qdq import mxfp4_qdq

    assert _native.device_status(clear=True) == 0
    _native.call("qdq_selftest_bounded_wait", 20_000_000, _native.stream_ptr(cuda_device))
    status = _native.device_status(clear=False)
    assert status == (TIMEOUT << 16) | SITE, hex(status)
    assert _native.device_status(clear=True) == status
    assert _native.device_status(clear=False) == 0
    # the context is still usable
    x = torch.randn(64, 256).to(torch.bfloat16)
    y = mxfp4_qdq(x.to(cuda_device)).cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(y, oq.mxfp4_qdq(x.view(torch.int16).numpy().view(np.uint16)))


def test_selftest_rejects_bad_timeouts():
    from vllm_qdq_plugin import _native
    with pytest.raises(_native.NativeError):
        _native.call("qdq_selftest_bounded_wait", 0, None)
