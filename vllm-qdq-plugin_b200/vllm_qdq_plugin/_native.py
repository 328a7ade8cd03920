# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of `libqdq_b200.so` and the torch.library ops built on it.

The C ABI (include/qdq_b200.h) takes raw device pointers, element strides and
a `cudaStream_t`; this module passes `tensor.data_ptr()` and torch's current
stream, so the kernels are stream-ordered with the caller's other work and no
host synchronisation happens.  There is no CPU fallback: a CPU tensor or a
missing library raises.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

DTYPE_CODE = {torch.bfloat16: 0, torch.float16: 1}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes (restype is always c_int status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "qdq_mxfp4": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64,
                  _int, _int, _c_void_p],
    "qdq_mxfp8": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64,
                  _int, _int, _c_void_p],
    "qdq_nvfp4": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64,
                  _i64, _int, _c_void_p],
    "qdq_nvfp4_global_scale": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _int,
                               _c_void_p],
    "qdq_host_stream": [_int, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _int, _c_void_p,
                        _i64, _i64, _c_void_p],
    "qdq_host_stream_staging_bytes": [_i64, _i64, _int, _int],
    "qdq_last_error": [],
    "qdq_abi_version": [],
    "qdq_device_status": [ctypes.POINTER(ctypes.c_int), _int],
    "qdq_selftest_bounded_wait": [_i64, _c_void_p],
    "sage3_attn_workspace_bytes": [_i64, _i64, _i64, _i64],
    "sage3_fp4_attn": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64,
                       ctypes.POINTER(ctypes.c_int64), _f32, _int, _int, _int, _int, _int, _c_void_p,
                       _i64, _c_void_p],
    "fp4_moe_mxf4": [_c_void_p, _i64, _int, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p,
                     _c_void_p, _i64, _int, _int, _int, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _i64,
                     _c_void_p],
    "fp4_moe_workspace_bytes": [_i64, _int, _i64],
    "qdq_sf_tiled_bytes": [_i64, _i64],
    "qdq_sf_tile": [_c_void_p, _c_void_p, _i64, _i64, _i64, _int, _c_void_p],
    "fp4_gemm_mxf4": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64,
                      _i64, _i64, _i64, _i64, _int, _c_void_p],
    "fp4_linear_workspace_bytes": [_i64, _i64],
    "qdq_sf16_tiled_bytes": [_i64, _i64],
    "fp4_gemm_nvf4": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p,
                      _i64, _i64, _i64, _i64, _i64, _i64, _int, _c_void_p],
    "fp4_linear_nvf4_workspace_bytes": [_i64, _i64],
    "fp4_linear_nvf4": [_c_void_p, _i64, _int, _c_void_p, _c_void_p, _c_void_p, _f32, _c_void_p, _c_void_p,
                        _i64, _i64, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
    "fp4_linear_noalloc_scratch_bytes": [],
    "fp4_linear_mxf4_noalloc": [_c_void_p, _i64, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                _i64, _i64, _i64, _i64, _i64, _c_void_p],
    "fp4_linear_mxf4": [_c_void_p, _i64, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64,
                        _i64, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p],
}
_RESTYPES = {"qdq_last_error": ctypes.c_char_p, "qdq_sf_tiled_bytes": ctypes.c_int64,
             "fp4_linear_workspace_bytes": ctypes.c_int64,
             "qdq_sf16_tiled_bytes": ctypes.c_int64,
             "fp4_linear_nvf4_workspace_bytes": ctypes.c_int64,
             "fp4_linear_noalloc_scratch_bytes": ctypes.c_int64,
             "sage3_attn_workspace_bytes": ctypes.c_int64,
             "fp4_moe_workspace_bytes": ctypes.c_int64,
             "qdq_host_stream_staging_bytes": ctypes.c_int64}


def lib() -> ctypes.CDLL:
    """Load (building first if missing or stale) the sm_100a library."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.build_native()
            handle = ctypes.CDLL(str(path))
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _LIB = handle
    return _LIB


def library_path() -> str:
    return str(_build.LIB_PATH)


class NativeError(RuntimeError):
    """A C-ABI entry point returned a non-zero qdq_status_t."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


def check(fn: str, status: int) -> None:
    if status != 0:
        msg = lib().qdq_last_error()
        raise NativeError(fn, status, msg.decode() if msg else "")


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def device_status(clear: bool = True) -> int:
    """The library's device status word (0 = ok; else (status << 16) | site)."""
    out = ctypes.c_int(0)
    call("qdq_device_status", ctypes.byref(out), int(clear))
    return out.value


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "vllm_qdq_plugin (B200) kernels need CUDA tensors on an sm_100 GPU; "
                f"got a tensor on {t.device} (there is no CPU fallback)")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()
