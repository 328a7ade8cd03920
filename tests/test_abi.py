"""CPU: the C-ABI library builds for sm_100a, loads, exports every symbol that
include/*.h declares, and rejects bad arguments before touching the GPU."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import REPO
from vllm_qdq_plugin import _build, _native

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "defined") and not name.isupper():
                names.add(name)
    return names


def test_headers_declare_the_entry_points():
    names = declared_symbols()
    for expect in ("qdq_mxfp4", "qdq_nvfp4", "qdq_nvfp4_global_scale", "qdq_last_error",
                   "qdq_abi_version"):
        assert expect in names


def test_library_exports_every_declared_symbol():
    path = _build.build_native()
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared_symbols() - exported
    assert not missing, f"declared in include/*.h but not exported: {sorted(missing)}"
    lib = ctypes.CDLL(str(path))
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_build_targets_sm100a_only():
    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "--use_fast_math" not in _build.NVCC_FLAGS


def test_abi_version_and_argument_errors_without_gpu():
    lib = _native.lib()
    assert lib.qdq_abi_version() >= 100
    # group size other than 32 is refused before any CUDA call
    st = lib.qdq_mxfp4(1, 1, None, None, 4, 64, 64, 64, 0, 16, None)
    assert st == 2 and b"group_size" in lib.qdq_last_error()
    st = lib.qdq_mxfp4(None, 1, None, None, 4, 64, 64, 64, 0, 32, None)
    assert st == 1 and b"null" in lib.qdq_last_error()
    st = lib.qdq_mxfp4(1, 1, None, None, 4, 64, 64, 64, 7, 32, None)
    assert st == 1 and b"dtype" in lib.qdq_last_error()
    st = lib.qdq_mxfp4(1, 1, None, None, -1, 64, 64, 64, 0, 32, None)
    assert st == 1
    st = lib.qdq_mxfp4(1, 1, None, None, 4, 64, 32, 64, 0, 32, None)
    assert st == 1 and b"stride" in lib.qdq_last_error()
    st = lib.qdq_mxfp4(1, 1, None, None, 4, 64, 64, 128, 0, 32, None)  # in place needs ldx == ldy
    assert st == 1
    # empty tensors are a no-op success
    assert lib.qdq_mxfp4(1, 2, None, None, 0, 64, 64, 64, 0, 32, None) == 0
    st = lib.qdq_nvfp4(1, 2, None, None, 3, 4, 40, 40, 40, 0, None)
    assert st == 1 and b"multiple of 16" in lib.qdq_last_error()
    st = lib.qdq_nvfp4(1, 2, None, None, None, 4, 64, 64, 64, 0, None)
    assert st == 1 and b"global_scale" in lib.qdq_last_error()
    st = lib.qdq_nvfp4_global_scale(1, 2, 3, 0, 64, 64, 0, None)
    assert st == 1


def test_native_error_is_raised_with_message():
    with pytest.raises(_native.NativeError, match="group_size"):
        _native.call("qdq_mxfp4", 1, 1, None, None, 4, 64, 64, 64, 0, 16, None)


def test_cpu_tensors_are_rejected_loudly():
    import torch
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        mxfp4_qdq(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        nvfp4_qdq(x, global_scale=torch.ones(1))


def test_reference_assertions_are_kept():
    import torch
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    with pytest.raises(AssertionError, match="2D"):
        mxfp4_qdq(torch.zeros(2, 3, 64, dtype=torch.bfloat16))
    with pytest.raises(AssertionError, match="fp16/bf16"):
        mxfp4_qdq(torch.zeros(2, 64, dtype=torch.float32))


def test_host_streaming_qdq_checks_its_arguments_before_touching_a_gpu():
    import torch
    from vllm_qdq_plugin.qdq import qdq_from_host
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="global_scale"):
        qdq_from_host(x, "nvfp4")
    with pytest.raises(ValueError, match="unknown format"):
        qdq_from_host(x, "int4")
    with pytest.raises(AssertionError, match="fp16/bf16"):
        qdq_from_host(x.float(), "mxfp4")
    with pytest.raises(ValueError, match="out must be"):
        qdq_from_host(x, "mxfp4", out=torch.zeros(4, 32, dtype=torch.bfloat16))


def test_host_stream_format_codes_match_the_header():
    import re
    from vllm_qdq_plugin.qdq import host
    header = (REPO / "include" / "qdq_b200.h").read_text()
    codes = {m.group(1).lower(): int(m.group(2))
             for m in re.finditer(r"QDQ_FORMAT_(\w+)\s*=\s*(\d+)", header)}
    assert codes == host._FORMATS
