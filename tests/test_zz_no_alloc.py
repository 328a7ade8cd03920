"""The allocation-free fused FP4 linear (fp4_linear_mxf4_noalloc).

Callers that cannot allocate device memory at the call site (an embedding C or
C++ host without an allocator, or an engine whose memory pool is fully
reserved) use this entry point; its activation scratch is a static array in
the library's device memory.  Through the C ABI, calls in a row must give
the same result as the workspace-taking fp4_linear_mxf4 (same kernels, so
bit-identical, which is inside the GEMM tests' tolerance).  Runs last so a
failure here leaves every other test already run; it also passes alone in a
fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _linear_with_workspace(lib, a, w, out):
    from vllm_qdq_plugin import _native
    m, k = a.shape
    ws = torch.empty((lib.fp4_linear_workspace_bytes(m, k),), dtype=torch.uint8, device=a.device)
    _native.call("fp4_linear_mxf4", a.data_ptr(), k, 0, w.codes.data_ptr(), w.sf_tiled.data_ptr(),
                 None, out.data_ptr(), m, w.n, k, k // 2, w.n, ws.data_ptr(), ws.numel(),
                 _native.stream_ptr(a.device))


def _linear_noalloc(a, w, out):
    from vllm_qdq_plugin import _native
    m, k = a.shape
    _native.call("fp4_linear_mxf4_noalloc", a.data_ptr(), k, 0, w.codes.data_ptr(),
                 w.sf_tiled.data_ptr(), None, out.data_ptr(), m, w.n, k, k // 2, w.n,
                 _native.stream_ptr(a.device))


def test_noalloc_linear_matches_workspace_linear_twice(cuda_device):
    from oracle import gemm as og
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.gemm import prepare_mxfp4_weight
    lib = _native.lib()
    results = []
    # The third call has K % 256 != 0 (row-major scales, then a separate
    # scale-tiling launch) and fewer rows than the call before it, so it runs
    # over scratch that still holds the larger call's codes and scales.
    for call, (m, n, k, seed) in enumerate([(300, 512, 2048, 5), (1024, 768, 4096, 6), (300, 384, 2080, 7)]):
        g = torch.Generator().manual_seed(seed)
        a = torch.randn(m, k, generator=g).to(torch.bfloat16).to(cuda_device)
        codes, scales = og.random_mxfp4_weight(n, k, seed)
        w = prepare_mxfp4_weight(torch.from_numpy(codes).to(cuda_device),
                                 torch.from_numpy(scales).to(cuda_device))
        want = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        _linear_with_workspace(lib, a, w, want)
        _linear_noalloc(a, w, got)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"call {call}"
        results.append(got)
    assert _native.device_status() == 0


def test_noalloc_rejects_oversized_scratch(cuda_device):
    from vllm_qdq_plugin import _native
    lib = _native.lib()
    cap = lib.fp4_linear_noalloc_scratch_bytes()
    assert cap == 32 << 20
    m, k = 65536, 4096
    assert lib.fp4_linear_workspace_bytes(m, k) > cap
    with pytest.raises(_native.NativeError, match="scratch"):
        _native.call("fp4_linear_mxf4_noalloc", 16, k, 0, 16, 16, None, 16, m, 256, k, k // 2, 256,
                     None)
