# SPDX-License-Identifier: Apache-2.0
"""Build of the sm_100a shared library `libqdq_b200.so` (C ABI in include/qdq_b200.h).

The library is compiled in-tree with nvcc (no torch headers, no JIT cache), so
the built `.so` sits next to this package and travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
PLUGIN_ROOT = PKG_DIR.parent                       # vllm-qdq-plugin_b200/
CSRC_DIR = PLUGIN_ROOT / "csrc"
INCLUDE_DIR = PLUGIN_ROOT.parent / "include"       # repo-level public header
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libqdq_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math / -ftz: bf16/fp32 subnormals must survive for bit-exact QDQ.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
    return sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libqdq_b200.so for sm_100a")


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")


def build_native(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu into one sm_100a shared library (idempotent).

    Each translation unit is compiled to an object file in parallel (one nvcc
    per source), then nvcc links the objects into the shared library."""
    if not force and not is_stale():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor

    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = LIB_DIR / f".obj.{os.getpid()}"
    obj_dir.mkdir(exist_ok=True)
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    jobs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        jobs.append((obj, [nvcc_path(), *ARCH_FLAGS, *compile_flags, f"-I{INCLUDE_DIR}", f"-I{CSRC_DIR}",
                           "-c", "-o", str(obj), str(src)]))
    try:
        with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
            for fut in [pool.submit(_run, cmd, verbose) for _, cmd in jobs]:
                fut.result()
        tmp = LIB_PATH.with_name(f".{LIB_PATH.name}.{os.getpid()}.tmp")
        _run([nvcc_path(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp),
              *[str(o) for o, _ in jobs]], verbose)
        os.replace(tmp, LIB_PATH)
    finally:
        shutil.rmtree(obj_dir, ignore_errors=True)
    return LIB_PATH
