"""Generate the golden fixtures under tests/golden/ by running the reference.

Run inside the build container, where the reference checkout and vLLM 0.22 are
importable (CPU only):

    python tests/golden/make_golden.py --reference /path/to/vllm-qdq-plugin

Each fixture is a compressed .npz of inputs and the reference's own outputs:
  mxfp4_bf16.npz / mxfp4_fp16.npz   reference mxfp4_qdq (src/vllm_qdq_plugin/qdq/mxfp4.py:98)
                                    on every finite 16-bit pattern in natural 32-groups, on
                                    "context" groups (one large element fixing the scale plus
                                    smaller ones), on a config-1 slice and on odd K.
  nvfp4_bf16.npz / nvfp4_fp16.npz   vLLM 0.22 ref_nvfp4_quant_dequant, CPU branch
                                    (nvfp4_emulation_utils.py:455-478), same pattern sets,
                                    several global scales, and a config-2 slice.
  mxfp4_hw_quant.npz                reference quantize_to_mxfp4 (sage3/mxfp4_hw_kernel.py:73)
                                    codes and E8M0 bytes for Q/K-like and V-like rows.
  mxfp8_hw_quant.npz                reference quantize_to_mxfp8 (sage3/mxfp8_hw_kernel.py:37)
                                    E4M3 codes and E8M0 bytes for Q/K-like and V-like rows.
  mxfp8_bf16.npz / mxfp8_fp16.npz   reference mxfp8_qdq (src/vllm_qdq_plugin/qdq/mxfp8.py:73)
                                    on every finite 16-bit pattern in natural 32-groups, on
                                    context groups reaching 20 binades below their max (into
                                    E4M3's subnormal range), on a config-1 slice and on odd K.
The reference is imported from its checkout; nothing from it is copied here.
"""

from __future__ import annotations

import argparse
import ast
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from bench import c1_input, c2_input, global_scale_of  # noqa: E402


def load_reference(ref_root: Path):
    spec = importlib.util.spec_from_file_location(
        "ref_mxfp4", ref_root / "src/vllm_qdq_plugin/qdq/mxfp4.py")
    mx = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mx)
    sys.path.insert(0, str(ref_root / "src/vllm_qdq_plugin/sage3_attn"))
    from sage3 import mxfp4_hw_kernel  # noqa: E402  (reference package, CPU-safe parts)
    from vllm.model_executor.layers.quantization.utils import nvfp4_emulation_utils as nv
    return mx.mxfp4_qdq, nv.ref_nvfp4_quant_dequant, mxfp4_hw_kernel.quantize_to_mxfp4


def load_reference_mxfp8(ref_root: Path):
    spec = importlib.util.spec_from_file_location(
        "ref_mxfp8", ref_root / "src/vllm_qdq_plugin/qdq/mxfp8.py")
    m8 = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m8)
    return m8.mxfp8_qdq


def load_reference_mxfp8_hw(ref_root: Path):
    """quantize_to_mxfp8 from the reference's mxfp8_hw_kernel.py.  Importing the
    module asks Triton for an active GPU driver, so only the two CPU-safe
    functions it needs are compiled from the reference file here and run."""
    path = ref_root / "src/vllm_qdq_plugin/sage3_attn/sage3/mxfp8_hw_kernel.py"
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef)
            and n.name in ("fp8e8m0_to_float32", "quantize_to_mxfp8")]
    assert len(keep) == 2
    ns = {"torch": torch}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(path), "exec"), ns)
    return ns["quantize_to_mxfp8"]


def write_mxfp8_hw(ref_root: Path):
    quantize_to_mxfp8 = load_reference_mxfp8_hw(ref_root)
    g = torch.Generator().manual_seed(98)
    qk = (torch.randn(512, 128, generator=g) * torch.exp(torch.randn(512, 1, generator=g) * 3)
          ).to(torch.bfloat16).float()
    qk[7] = 0.0                                     # all-zero group: amax clamped to 1e-12
    qk[9, :32] = torch.tensor([2.0 ** -40] * 32)    # tiny values (E4M3 subnormal / zero codes)
    qk[11, :32] = -(2.0 ** -30)                     # tiny negatives under a large max: -0 codes
    qk[11, 0] = -1.0
    qk[13, 0] = 448.0                               # amax / 448 an exact power of two
    qk[15, 0] = 450.0                               # just above: the exponent bumps
    v = (torch.randn(128, 1024, generator=g) * 3).to(torch.bfloat16).float()
    out = {}
    for name, t in (("qk", qk), ("v", v)):
        codes, scales = quantize_to_mxfp8(t)
        out[f"{name}_x"] = t.numpy()
        out[f"{name}_codes"] = codes.view(torch.uint8).numpy()
        out[f"{name}_scales"] = scales.numpy()
    np.savez_compressed(HERE / "mxfp8_hw_quant.npz", **out)
    print("wrote mxfp8_hw_quant.npz")


def finite_patterns(fp16: bool) -> np.ndarray:
    p = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    if fp16:
        nan = ((p & 0x7C00) == 0x7C00) & ((p & 0x03FF) != 0)
    else:
        nan = ((p & 0x7F80) == 0x7F80) & ((p & 0x007F) != 0)
    return p[~nan]


def group_rows(vals: np.ndarray, g: int) -> np.ndarray:
    pad = (-len(vals)) % g
    return np.concatenate([vals, np.zeros(pad, np.uint16)]).reshape(-1, g)


def context_rows(fp16: bool, g: int, rng: np.random.Generator, binades: int = 10) -> np.ndarray:
    """Groups whose largest element is a chosen 'context' value and whose other
    elements sweep every pattern within `binades` binades below it."""
    mbits = 10 if fp16 else 7
    if fp16:
        ctx = [0x0001, 0x00FF, 0x02FF, 0x0300, 0x03FF, 0x0400, 0x3C00, 0x3E00, 0x3EFF, 0x3F00,
               0x3FFF, 0x4600, 0x5BFF, 0x5C00, 0x7BFF, 0x7AFF, 0x7B00, 0x1000, 0x2345, 0x6789]
    else:
        ctx = [0x0001, 0x001F, 0x005F, 0x0060, 0x007F, 0x0080, 0x3F80, 0x3FC0, 0x3FDF, 0x3FE0,
               0x3FFF, 0x40C0, 0x7F5F, 0x7F60, 0x7F7F, 0x2000, 0x1234, 0x5678, 0x00C0, 0x6000]
    rows = []
    for c in ctx:
        ef = c >> mbits
        lo = max(0, ef - binades) << mbits
        cand = np.arange(lo, c + 1, dtype=np.uint32).astype(np.uint16)
        cand = np.concatenate([cand, cand | 0x8000]).astype(np.uint16)
        rng.shuffle(cand)
        cand = cand[:4096]  # fp16 has 8x the mantissas of bf16: keep the fixture small
        body = group_rows(cand, g - 1)
        head = np.full((body.shape[0], 1), c, np.uint16)
        head[rng.random(body.shape[0]) < 0.5] |= 0x8000
        rows.append(np.concatenate([head, body], axis=1))
    return np.concatenate(rows)


def as_t(bits: np.ndarray, fp16: bool) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.float16 if fp16 else torch.bfloat16)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference plugin (vllm-qdq-plugin)")
    ap.add_argument("--only", choices=["all", "mxfp8", "mxfp8_hw"], default="all")
    args = ap.parse_args()
    if args.only in ("all", "mxfp8_hw"):
        write_mxfp8_hw(Path(args.reference))
    if args.only == "mxfp8_hw":
        return
    write_mxfp8(Path(args.reference))
    if args.only == "mxfp8":
        return
    mxfp4_qdq, nvfp4_qdq, quantize_to_mxfp4 = load_reference(Path(args.reference))
    rng = np.random.default_rng(1234)

    for fp16 in (False, True):
        tag = "fp16" if fp16 else "bf16"
        pats = finite_patterns(fp16)
        # ---- MXFP4
        sets = {
            "natural": group_rows(pats, 32),
            "context": context_rows(fp16, 32, rng),
        }
        c1 = bits_of(c1_input()[:16].to(torch.float16 if fp16 else torch.bfloat16))
        sets["c1_slice"] = c1
        g_odd = torch.Generator().manual_seed(7)
        sets["odd_k"] = bits_of((torch.randn(7, 100, generator=g_odd) * 3).to(
            torch.float16 if fp16 else torch.bfloat16))
        out = {}
        for name, xb in sets.items():
            out[f"{name}_x"] = xb
            out[f"{name}_y"] = bits_of(mxfp4_qdq(as_t(xb, fp16), group_size=32))
        np.savez_compressed(HERE / f"mxfp4_{tag}.npz", **out)
        # ---- NVFP4
        out = {}
        nat16 = group_rows(pats, 16)
        ctx16 = context_rows(fp16, 16, rng)
        gss = [1.0, 2688.0, 2.6880, 0.01, 1.0e6, 448.0 * 6.0 / 65504.0]
        for i, gs in enumerate(gss):
            g = torch.tensor([gs], dtype=torch.float32)
            for name, xb in (("natural", nat16), ("context", ctx16)):
                if fp16 and name == "natural" and i >= 3:
                    continue
                out[f"{name}_gs{i}_x"] = xb
                out[f"{name}_gs{i}_y"] = bits_of(nvfp4_qdq(as_t(xb, fp16), g, 16))
            out[f"gs{i}"] = np.array([gs], np.float32)
        full = c2_input()
        gs_full = global_scale_of(full)
        c2 = full[:8].to(torch.float16 if fp16 else torch.bfloat16)
        out["c2_slice_x"] = bits_of(c2)
        out["c2_slice_gs"] = gs_full.numpy()
        out["c2_slice_y"] = bits_of(nvfp4_qdq(c2, gs_full, 16))
        np.savez_compressed(HERE / f"nvfp4_{tag}.npz", **out)
        print(f"wrote mxfp4_{tag}.npz, nvfp4_{tag}.npz")

    # ---- quantize_to_mxfp4 (Q/K along D, V along N after the reference's permute)
    g = torch.Generator().manual_seed(99)
    qk = (torch.randn(512, 128, generator=g) * torch.exp(torch.randn(512, 1, generator=g) * 2)
          ).to(torch.bfloat16).float()
    v = (torch.randn(128, 1024, generator=g) * 3).to(torch.bfloat16).float()
    out = {}
    for name, t in (("qk", qk), ("v", v)):
        codes, scales = quantize_to_mxfp4(t)
        out[f"{name}_x"] = t.numpy()
        out[f"{name}_codes"] = codes.numpy()
        out[f"{name}_scales"] = scales.numpy()
    np.savez_compressed(HERE / "mxfp4_hw_quant.npz", **out)
    print("wrote mxfp4_hw_quant.npz")


def write_mxfp8(ref_root: Path):
    mxfp8_qdq = load_reference_mxfp8(ref_root)
    rng = np.random.default_rng(808)
    for fp16 in (False, True):
        tag = "fp16" if fp16 else "bf16"
        dt = torch.float16 if fp16 else torch.bfloat16
        sets = {
            "natural": group_rows(finite_patterns(fp16), 32),
            "context": context_rows(fp16, 32, rng, binades=20),
            "c1_slice": bits_of(c1_input()[:16].to(dt)),
        }
        g_odd = torch.Generator().manual_seed(8)
        sets["odd_k"] = bits_of((torch.randn(7, 100, generator=g_odd) * 3).to(dt))
        out = {}
        for name, xb in sets.items():
            out[f"{name}_x"] = xb
            out[f"{name}_y"] = bits_of(mxfp8_qdq(as_t(xb, fp16), group_size=32))
        np.savez_compressed(HERE / f"mxfp8_{tag}.npz", **out)
        print(f"wrote mxfp8_{tag}.npz")


if __name__ == "__main__":
    main()
