"""numpy front end of the C oracle (oracle/qdq_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() (as the
checker) and bench.py's CPU-baseline / reference arm.  The product path under
vllm-qdq-plugin_b200/ never imports this.

Arrays of bf16/fp16 values are passed as uint16 bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "qdq_oracle.c"
LIB = HERE / "liboracle.so"
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        tmp = LIB.with_name(f".liboracle.{os.getpid()}.so")
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
                        "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                h = ctypes.CDLL(str(build()))
                vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
                h.oracle_mxfp4_qdq.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32]
                h.oracle_mxfp4_qdq.restype = None
                h.oracle_nvfp4_qdq.argtypes = [vp, vp, vp, vp, f32, i64, i64, i64, i64, i32, i32]
                h.oracle_nvfp4_qdq.restype = None
                h.oracle_nvfp4_global_scale.argtypes = [vp, i64, i64, i64, i32]
                h.oracle_nvfp4_global_scale.restype = f32
                h.oracle_round_e4m3.argtypes = [f32]
                h.oracle_round_e4m3.restype = f32
                h.oracle_mxfp4_hw_quant.argtypes = [vp, vp, vp, i64, i64, i32]
                h.oracle_mxfp4_hw_quant.restype = None
                h.oracle_mxfp8_hw_quant.argtypes = [vp, vp, vp, i64, i64, i32]
                h.oracle_mxfp8_hw_quant.restype = None
                h.oracle_mxfp8_qdq.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, i32]
                h.oracle_mxfp8_qdq.restype = None
                h.oracle_max_threads.argtypes = []
                h.oracle_max_threads.restype = i32
                _lib = h
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def mxfp4_qdq(x: np.ndarray, *, fp16: bool = False, codes: bool = False, nthreads: int = 0):
    """x: uint16 [M, K] bit patterns -> y (uint16 [M, K]) [, codes, scales]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = x.shape
    y = np.empty_like(x)
    kp = (k + 31) // 32 * 32
    c = np.empty((m, kp // 2), np.uint8) if codes else None
    s = np.empty((m, kp // 32), np.uint8) if codes else None
    lib().oracle_mxfp4_qdq(_p(x), _p(y), _p(c), _p(s), m, k, k, k, int(fp16), nthreads)
    return (y, c, s) if codes else y


def mxfp8_qdq(x: np.ndarray, *, fp16: bool = False, codes: bool = False, group_size: int = 32,
              nthreads: int = 0):
    """x: uint16 [M, K] bit patterns -> y (uint16 [M, K]) [, E4M3 codes [M, K], E8M0 scales]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = x.shape
    y = np.empty_like(x)
    c = np.empty((m, k), np.uint8) if codes else None
    s = np.empty((m, (k + group_size - 1) // group_size), np.uint8) if codes else None
    lib().oracle_mxfp8_qdq(_p(x), _p(y), _p(c), _p(s), m, k, k, k, int(fp16), group_size, nthreads)
    return (y, c, s) if codes else y


def nvfp4_qdq(x: np.ndarray, gs: float, *, fp16: bool = False, codes: bool = False,
              nthreads: int = 0):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = x.shape
    assert k % 16 == 0
    y = np.empty_like(x)
    c = np.empty((m, k // 2), np.uint8) if codes else None
    s = np.empty((m, k // 16), np.uint8) if codes else None
    lib().oracle_nvfp4_qdq(_p(x), _p(y), _p(c), _p(s), float(gs), m, k, k, k, int(fp16),
                           nthreads)
    return (y, c, s) if codes else y


def nvfp4_global_scale(x: np.ndarray, *, fp16: bool = False) -> float:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    m, k = x.shape
    return float(lib().oracle_nvfp4_global_scale(_p(x), m, k, k, int(fp16)))


def round_e4m3(v: float) -> float:
    return float(lib().oracle_round_e4m3(float(v)))


def mxfp4_hw_quant(x: np.ndarray, nthreads: int = 0):
    """quantize_to_mxfp4 restated: fp32 [..., K] -> (codes [..., K/2], scales [..., K/32])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    assert k % 32 == 0
    rows = x.size // k
    c = np.empty(x.shape[:-1] + (k // 2,), np.uint8)
    s = np.empty(x.shape[:-1] + (k // 32,), np.uint8)
    lib().oracle_mxfp4_hw_quant(_p(x), _p(c), _p(s), rows, k, nthreads)
    return c, s


def mxfp8_hw_quant(x: np.ndarray, nthreads: int = 0):
    """quantize_to_mxfp8 restated: fp32 [..., K] -> (E4M3 bytes [..., K], E8M0 scales [..., K/32])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    assert k % 32 == 0
    rows = x.size // k
    c = np.empty(x.shape, np.uint8)
    s = np.empty(x.shape[:-1] + (k // 32,), np.uint8)
    lib().oracle_mxfp8_hw_quant(_p(x), _p(c), _p(s), rows, k, nthreads)
    return c, s


def max_threads() -> int:
    return int(lib().oracle_max_threads())
