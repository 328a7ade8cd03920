#!/usr/bin/env python
"""Benchmark of the B200 FP4 hot path (one JSON line on rank 0).

Default run (no --workload): the headline is BASELINE config 2, the config the
QDQ metric is quoted on: NVFP4 activation QDQ of a bf16 [16384, 8192] tensor
(groups of 16, E4M3 block scales, fp32 global scale gs = 2688/amax).  A
"step" is one QDQ pass over that tensor.  The same line carries
`sub_records`, each measured in the same run the same way (device time,
roofline, clocks, end-to-end through the public API):
  config 1   MXFP4 QDQ bf16 [8192, 4096]
  config 3   QDQ fused into the tcgen05 FP4 GEMM, M = 4096 and the M = 16
             decode shape, beside vLLM's QDQ + Marlin timed on the same GPU
  config 4   Sage3 mxfp4_hw attention, Wan-2.1 720p [1, 75600, 40, 128]
  config 5   Sage3 nvfp4 (bf16_pv_only) attention, Flux batch [8, 4608, 24, 128]
`--workload NAME` runs one workload alone (see WORKLOADS).

Arms:
  default            the sm_100a kernels through the C ABI (value) and through
                     the public plugin API with pinned host buffers (e2e)
  --impl reference   the reference's CPU algorithm (the C restatement under
                     oracle/, all host threads) on the same config and metric

Multi-GPU (torchrun, one process per GPU): strong scaling.  The job is fixed
(config 2's 16384 rows; config 3's 4096 rows, or for M = 16 its 14336 output
columns; config 4's 40 heads; config 5's 8 batches) and each rank takes a
contiguous share of its units (vllm_qdq_plugin.shard).  No collective touches
the data path: the NVFP4 global scale is agreed by one fp32 all-reduce MIN
before timing, times are the max over ranks, and outputs are gathered over
NCCL only to verify them.  A `weak_scaling` sub-record repeats config 2 with
a full tensor per rank.
"""

from __future__ import annotations

import argparse
import ctypes
import contextlib
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "vllm-qdq-plugin_b200"))

import torch  # noqa: E402

BYTES_PER_ELT = 4  # 2 B read + 2 B written per bf16 element (algorithmic)
L2_BYTES = 126 * 1000 * 1000  # B200 L2 capacity
PUBLISHED_MS = {"mxfp4_hw": 261.81, "mxfp8_hw": 258.42, "sdpa_bf16": 84.56}  # reference, 1x B200, config 4

# ---------------------------------------------------------------------------
# seeded synthetic inputs (shapes and distributions of the BASELINE configs)
# ---------------------------------------------------------------------------


def c1_input(rows: int = 8192, cols: int = 4096, seed: int = 0) -> torch.Tensor:
    """Config 1: N(0,1) with 0.1% of positions (seeded) scaled by 50, bf16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    n = x.numel()
    idx = torch.randperm(n, generator=g)[: n // 1000]
    x.view(-1)[idx] *= 50.0
    return x.to(torch.bfloat16)


def c2_input(rows: int = 16384, cols: int = 8192, seed: int = 1) -> torch.Tensor:
    """Config 2: N(0,1) times per-row magnitudes log-uniform in [0.01, 100], bf16."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    lo, hi = math.log(0.01), math.log(100.0)
    mag = torch.exp(torch.rand(rows, 1, generator=g) * (hi - lo) + lo)
    return (x * mag).to(torch.bfloat16)


def global_scale_of(x: torch.Tensor) -> torch.Tensor:
    """gs = 448*6 / amax(|x|) in fp32 (vLLM's multiplier convention)."""
    amax = x.abs().max().to(torch.float32)
    return (torch.tensor(2688.0, dtype=torch.float32) / amax).reshape(1)


def c3_inputs(rows: int = 4096, n: int = 14336, k: int = 4096):
    """Config 3: A ~ N(0,1) bf16 [M, K] (seed 2); W MXFP4 [N, K]: uniform random
    E2M1 nibbles, E8M0 exponents uniform in [-10, -4] per 32-group (seed 3)."""
    import numpy as np
    g = torch.Generator().manual_seed(2)
    a = torch.randn(rows, k, generator=g).to(torch.bfloat16)
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    scales = (127 + rng.integers(-10, -3, size=(n, k // 32))).astype(np.uint8)
    return a, torch.from_numpy(codes), torch.from_numpy(scales)


def c4_inputs(dev, L: int = 75600, H: int = 40, seed: int = 4):
    """Config 4: Q, V ~ N(0,1); K ~ N(0,1) + a per-channel offset ~ N(0,3) of
    shape [1, 1, H, D] shared across tokens; NHD bf16 (generated on the device)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(1, L, H, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, L, H, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k += (torch.randn(1, 1, H, 128, generator=g, device=dev) * 3.0).to(torch.bfloat16)
    v = torch.randn(1, L, H, 128, generator=g, device=dev, dtype=torch.bfloat16)
    return q, k, v


def c5_inputs(dev, B: int = 8, L: int = 4608, H: int = 24, seed: int = 5):
    """Config 5: Q/K/V ~ N(0,1) NHD bf16; 1% of K rows of every (b, h), chosen
    per (b, h) with the seeded generator, scaled by 20."""
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, L, H, 128, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, L, H, 128, generator=g, device=dev)
    pick = torch.rand(B, L, H, 1, generator=g, device=dev).argsort(dim=1) < (L // 100)
    k = torch.where(pick, k * 20.0, k).to(torch.bfloat16)
    v = torch.randn(B, L, H, 128, generator=g, device=dev, dtype=torch.bfloat16)
    return q, k, v


def moe_inputs(m: int, e: int, top_k: int, n: int, k: int, seed: int = 6):
    """Synthetic MoE layer: A ~ N(0,1) bf16 [m, k]; per-expert MXFP4 weights with
    uniform nibbles and E8M0 exponents in [-10, -4]; each token routed to top_k
    distinct experts uniformly; routing weights U(0, 1); block size 64 (16 when
    fewer than 32 slots per expert on average)."""
    import numpy as np
    sys.path.insert(0, str(REPO))
    from oracle import gemm as og  # moe_align: vLLM's moe_align_block_size layout
    rng = np.random.default_rng(seed)
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    codes = torch.from_numpy(rng.integers(0, 256, size=(e, n, k // 2), dtype=np.uint8))
    scales = torch.from_numpy((127 + rng.integers(-10, -3, size=(e, n, k // 32))).astype(np.uint8))
    topk_ids = np.argsort(rng.random((m, e)), axis=1)[:, :top_k]
    bs = 64 if m * top_k >= 32 * e else 16
    sid, eid, ntp = og.moe_align(topk_ids, e, bs)
    topk_w = torch.from_numpy(rng.random((m, top_k)).astype(np.float32))
    return a, codes, scales, torch.from_numpy(sid), torch.from_numpy(eid), torch.from_numpy(ntp), topk_w, bs


WORKLOADS = {
    "nvfp4_qdq": dict(config="BASELINE config 2: NVFP4 QDQ bf16 [16384, 8192], group 16, "
                             "E4M3 block scales, fp32 gs = 2688/amax",
                      rows=16384, cols=8192, make=c2_input),
    "mxfp4_qdq": dict(config="BASELINE config 1: MXFP4 QDQ bf16 [8192, 4096], group 32, E8M0",
                      rows=8192, cols=4096, make=c1_input),
    "mxfp8_qdq": dict(config="MXFP8 QDQ (float8_e4m3fn Marlin layers) on the config-1 input: bf16 "
                             "[8192, 4096], group 32, E8M0 scales, E4M3 elements",
                      rows=8192, cols=4096, make=c1_input),
    "sage3_mxfp4": dict(config="BASELINE config 4: Sage3 self-attention, MXFP4, Wan-2.1-14B 720p: "
                               "B=1, H=40, L=75600, D=128, bf16 NHD, non-causal, fp32 accumulation",
                        rows=75600, cols=128, B=1, H=40, sage3="mxfp4_hw", acc="fp32"),
    "sage3_mxfp8": dict(config="Sage3 self-attention, mxfp8_hw (E4M3 + E8M0 per 32), on BASELINE config 4's "
                               "shape: B=1, H=40, L=75600, D=128, bf16 NHD, non-causal, fp32 accumulation",
                        rows=75600, cols=128, B=1, H=40, sage3="mxfp8_hw", acc="fp32"),
    "sage3_nvfp4": dict(config="BASELINE config 5: Sage3 self-attention, NVFP4, SAGE3_ACC_DTYPE=bf16_pv_only, "
                               "Flux-like batch: B=8, H=24, L=4608, D=128, bf16 NHD, 1% of K rows x20",
                        rows=4608, cols=128, B=8, H=24, sage3="nvfp4", acc="bf16_pv_only"),
    "mxfp4_moe": dict(config="Grouped MXFP4 MoE GEMM (QDQ + moe_wna16_marlin_gemm replaced), gpt-oss-120b "
                             "w13 shape: 4096 tokens, 128 experts, top-4, K=2880, N=5760, block 64, "
                             "uniform routing", rows=4096, cols=2880, E=128, N=5760, top_k=4),
    "mxfp4_linear": dict(config="BASELINE config 3: MXFP4 QDQ fused into a tcgen05 FP4 GEMM, "
                                "A bf16 [M=4096, K=4096], W MXFP4 [N=14336, K=4096], out bf16",
                         rows=4096, cols=4096),
    "nvfp4_linear": dict(config="BASELINE config 3's shape with NVFP4 weights and activations (VLLM_QDQ_NVFP4_ACT): "
                                "A bf16 [M=4096, K=4096] -> E2M1 + E4M3 per 16 + gs = 2688/amax, W NVFP4 "
                                "[N=14336, K=4096] (E4M3 scales per 16, tensor scale 1/2048), out bf16",
                         rows=4096, cols=4096),
}

# ---------------------------------------------------------------------------
# environment helpers
# ---------------------------------------------------------------------------


def _peaks() -> dict:
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def measured_peak_hbm() -> tuple[float, str]:
    p = _peaks()
    if "hbm_gbs" in p:
        return float(p["hbm_gbs"]), "of measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "of fallback (6.65 TB/s)"


def measured_peak_fp8() -> tuple[float, str]:
    """Dense FP8 tensor peak: 2x the measured cuBLAS bf16 rate (4.5 vs 2.25 PFLOP/s nominal)."""
    p = _peaks()
    if "bf16_tflops" in p:
        return 2.0 * float(p["bf16_tflops"]), "of measured bf16 x 2 (MEASURED_PEAKS.json bf16_tflops)"
    return 2.0 * 1590.0, "of fallback bf16 1.59 PF x 2"


def measured_peak_fp4() -> tuple[float, str]:
    """Dense FP4 tensor peak: the sm_100 dense FP4 rate is 4x the bf16 rate
    (9 vs 2.25 PFLOP/s nominal); MEASURED_PEAKS.json has the cuBLAS bf16 figure."""
    p = _peaks()
    if "bf16_tflops" in p:
        return 4.0 * float(p["bf16_tflops"]), "of measured bf16 x 4 (MEASURED_PEAKS.json bf16_tflops)"
    return 4.0 * 1590.0, "of fallback bf16 1.59 PF x 4"


def ncu_traffic(key: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    try:
        return json.loads((REPO / "profiles" / "roofline_traffic.json").read_text())[key]["bytes_per_launch"]
    except Exception:
        return None


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi's first sample can take a second on a fresh box: wait for
        # it, so that the samples bracket even a timed region of a few ms
        deadline = time.time() + 5.0
        while not self.samples and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.02)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [f.strip() for f in line.split(",")]))

    def stop(self, after: float | None = None):
        if after is not None:  # one sample past the end of the timed region
            deadline = time.time() + 1.0
            while time.time() < deadline and not any(t > after for t, _ in self.samples):
                time.sleep(0.02)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float):
        if not self.samples:
            return None
        # samples inside the timed region; a region shorter than the 100 ms
        # sampling period has none, and then the samples next to it count
        inside = [s for t, s in self.samples if t0 <= t <= t1]
        window = inside or [s for t, s in self.samples if t0 - 0.25 <= t <= t1 + 0.25] or \
            [s for _, s in self.samples]
        mhz = [float(s[1]) for s in window if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in window if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in window for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(window), "samples_inside_timed_region": len(inside)}


# ---------------------------------------------------------------------------
# per-rank context and timing
# ---------------------------------------------------------------------------


@dataclasses.dataclass
class Ctx:
    world: int
    rank: int
    local: int
    dev: torch.device
    dist: object | None
    args: argparse.Namespace
    host_cpus: list | None = None  # CPUs this rank is pinned to (NVML's list for its GPU), None if unchanged
    all_cpus: set | None = None    # the CPUs the process started with (the CPU baselines use all of them)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def max_ms(self, ms: float) -> float:
        from vllm_qdq_plugin import shard
        return shard.max_over_ranks(ms, self.dev)

    def share(self, units: int) -> tuple[int, int]:
        from vllm_qdq_plugin import shard
        return shard.unit_range(units, self.rank, self.world)


def timed(ctx: Ctx, run, steps: int, graph: bool = True, clocks: bool = True):
    """Time `steps` calls of run(i, stream_ptr) on the device: captured once in
    a CUDA graph and replayed (graph=True), or issued eagerly.  Barriers and
    synchronisation bracket the timed region; the result is the max over
    ranks.  Returns (ms per step, clock summary of rank 0)."""
    stream = torch.cuda.current_stream(ctx.dev)
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(ctx.dev)
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            with torch.cuda.graph(g, stream=cap):
                for i in range(steps):
                    run(i, cap.cuda_stream)
        stream.wait_stream(cap)
        g.replay()  # the first replay uploads the graph
        ctx.barrier()

        def body():
            g.replay()
    else:
        def body():
            for i in range(steps):
                run(i, stream.cuda_stream)
    sampler = ClockSampler(ctx.local).start() if (ctx.rank == 0 and clocks) else None
    time.sleep(0.3 if sampler else 0)
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    # A ~100 us spin kernel ahead of the start event: the host submits the
    # steps while it runs, so the timed region holds the K steps themselves,
    # not the host's submission latency (about 29 us for a 20-node graph).
    torch.cuda._sleep(200_000)
    e0.record(stream)
    body()
    e1.record(stream)
    ctx.barrier()
    t1 = time.time()
    ms = ctx.max_ms(e0.elapsed_time(e1))
    summary = None
    if sampler:
        sampler.stop(after=t1)
        summary = sampler.summary(t0, t1)
    del g
    return ms / steps, summary


def timed_host(ctx: Ctx, step, steps: int) -> float:
    """Time `steps` end-to-end calls (host buffers in and out) with CUDA events
    on the current stream; max over ranks; ms per step."""
    stream = torch.cuda.current_stream(ctx.dev)
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    ctx.barrier()
    return ctx.max_ms(e0.elapsed_time(e1)) / steps


# ---------------------------------------------------------------------------
# CPU baselines (the oracle = the reference's algorithm restated; reported only)
# ---------------------------------------------------------------------------


@contextlib.contextmanager
def all_host_cpus(ctx: "Ctx"):
    """The CPU baselines run on every core the process started with, not only
    the GPU-local ones the rank is pinned to."""
    if not ctx.host_cpus or not ctx.all_cpus:
        yield
        return
    os.sched_setaffinity(0, ctx.all_cpus)
    try:
        yield
    finally:
        os.sched_setaffinity(0, ctx.host_cpus)


def cpu_baseline(workload: str, x: torch.Tensor, budget_s: float = 15.0) -> dict:
    """Reported baseline: the oracle (C restatement of the reference) on host cores."""
    sys.path.insert(0, str(REPO))
    from oracle import qdq as oq  # test/baseline infrastructure only

    cores = os.cpu_count() or 1
    xb = x.view(torch.int16).numpy().view("uint16")
    if workload == "nvfp4_qdq":
        gs = float(global_scale_of(x)[0])
        fn = lambda: oq.nvfp4_qdq(xb, gs, nthreads=cores)  # noqa: E731
    elif workload == "mxfp8_qdq":
        fn = lambda: oq.mxfp8_qdq(xb, nthreads=cores)  # noqa: E731
    else:
        fn = lambda: oq.mxfp4_qdq(xb, nthreads=cores)  # noqa: E731
    fn()
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n
    out = {"value": round(x.numel() * BYTES_PER_ELT / dt / 1e9, 3), "unit": "GB/s",
           "cores": cores, "kind": "port",
           "sample": f"{n} full passes over the [{x.shape[0]}, {x.shape[1]}] input "
                     "(C restatement of the reference algorithm, OpenMP)"}
    if workload == "nvfp4_qdq":
        out["vllm_torch_cpu"] = vllm_nvfp4_cpu(x)
    return out


def vllm_nvfp4_cpu(x: torch.Tensor, rows: int = 1024) -> dict | None:
    """The NVFP4 QDQ the reference's path is defined by, vLLM 0.22's torch
    emulation (nvfp4_emulation_utils.py:439-478 ref_nvfp4_quant, then its CPU
    branch's dequantise), on a sample of rows with all host threads."""
    try:
        from vllm.model_executor.layers.quantization.utils import nvfp4_emulation_utils as nv
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"vLLM import failed: {e}"}
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    xs = x[:rows].contiguous()
    gs = global_scale_of(x)

    def fn():
        q, bs = nv.ref_nvfp4_quant(xs, gs, 16)
        m, k = xs.shape
        return (q.reshape(m, k // 16, 16) * (bs.unsqueeze(-1) / gs)).reshape(m, k).to(xs.dtype)

    fn()
    t0 = time.perf_counter()
    n = 0
    while n < 3 or time.perf_counter() - t0 < 3.0:
        fn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(xs.numel() * BYTES_PER_ELT / dt / 1e9, 4), "unit": "GB/s", "cores": cores,
            "sample": f"first {rows} rows, {n} passes: vLLM ref_nvfp4_quant + its CPU dequantise (torch)"}


def cpu_gemm_sample(m: int, budget_s: float = 15.0, max_rows: int = 256) -> dict:
    """The reference's CPU emulation of the fused linear (mxfp4_qdq of the
    activation, then an fp32 matmul with the dequantised MXFP4 weight) on a
    sample of activation rows, all host threads; W is dequantised once
    beforehand (weight preparation)."""
    sys.path.insert(0, str(REPO))
    from oracle import gemm as og
    from oracle import qdq as oq  # test/baseline infrastructure only

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rows = min(m, max_rows)
    a, codes, scales = c3_inputs(rows=rows)
    n, k = codes.shape[0], codes.shape[1] * 2
    w = torch.from_numpy(og.dequant_mxfp4(codes.numpy(), scales.numpy()).astype("float32"))
    ab = a.view(torch.int16).numpy().view("uint16")

    def fn():
        aq = oq.mxfp4_qdq(ab, nthreads=cores)
        at = torch.from_numpy(aq.astype("int16")).view(torch.bfloat16).float()
        return (at @ w.t()).to(torch.bfloat16)

    fn()
    it, t0 = 0, time.perf_counter()
    while True:
        fn()
        it += 1
        if time.perf_counter() - t0 > budget_s or it >= 200:
            break
    dt = (time.perf_counter() - t0) / it
    return {"value": round(2.0 * rows * n * k / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"{rows} of {m} activation rows x W [{n}, {k}] per pass, {it} passes: C restatement "
                      "of mxfp4_qdq + torch fp32 matmul with the dequantised weight (W dequantised once)"}


def cpu_attn_sample(wl: dict, L: int, budget_s: float = 20.0) -> dict:
    """The reference's Sage3 path restated on the CPU (oracle/attn.py) for one
    (batch, head): its pre-pass over all L tokens, and the flash loop for as many
    128-row query tiles as fit the budget; the per-head time is extrapolated as
    pre-pass + (query tiles) x (time per tile)."""
    sys.path.insert(0, str(REPO))
    from oracle import attn as oa  # test/baseline infrastructure only

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    if wl["sage3"] == "nvfp4":
        q, k, v = c5_inputs(torch.device("cpu"), B=1, L=L, H=1)
    else:
        q, k, v = c4_inputs(torch.device("cpu"), L=L, H=1)
    f = lambda t: t[0, :, 0].float().numpy()  # noqa: E731
    qk_fmt, pv_fmt, emulated, pre, vsmooth, qk_smooth = oa.CONFIGS[wl["sage3"]]
    block_n = oa.REF_BLOCK_N[wl["sage3"]]
    sm = 1.0 / math.sqrt(128)
    t0 = time.perf_counter()
    qd, kd, vd, ds = oa.prepass(f(q), f(k), f(v), qk_smooth, qk_fmt=qk_fmt, pv_fmt=pv_fmt, vsmooth=vsmooth)
    t_pre = time.perf_counter() - t0
    tiles = (L + 127) // 128
    done, t0 = 0, time.perf_counter()
    while done < tiles:
        oa.flash(qd, kd, vd, ds, L, sm, block_n=block_n, emulated=emulated,
                 q_rows=slice(128 * done, 128 * done + 128), pre=pre, **oa.p_flags(pv_fmt))
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    t_tile = (time.perf_counter() - t0) / done
    per_head = t_pre + tiles * t_tile
    return {"value": round(4.0 * L * L * 128 / per_head / 1e12, 6), "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"one (batch, head) at L={L}: pre-pass {t_pre:.2f} s + {done} of {tiles} query tiles "
                      f"timed ({t_tile:.3f} s each), per-head time extrapolated to all tiles; numpy/C "
                      f"restatement of the reference's {wl['sage3']} path"}


def cpu_moe_sample(wl: dict, m: int, budget_s: float = 15.0) -> dict:
    """The reference's CPU emulation of the MoE layer (mxfp4_qdq of the gathered
    tokens, fp32 matmul with each dequantised expert) on a sample of experts,
    all host threads; extrapolated to every routed slot."""
    import numpy as np
    sys.path.insert(0, str(REPO))
    from oracle import gemm as og
    from oracle import qdq as oq  # test/baseline infrastructure only

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    e, n, k, top_k = wl["E"], wl["N"], wl["cols"], wl["top_k"]
    a, codes, scales, sid, eid, ntp, topk_w, bs = moe_inputs(m, e, top_k, n, k)
    sid, eid = sid.numpy(), eid.numpy()
    ab = a.view(torch.int16).numpy().view("uint16")
    done_slots, t0, ex = 0, time.perf_counter(), 0
    while ex < e:
        blocks = np.nonzero(eid == ex)[0]
        slots = np.concatenate([sid[b * bs:(b + 1) * bs] for b in blocks]) if len(blocks) else np.array([])
        slots = slots[slots < m * top_k]
        if len(slots):
            w = torch.from_numpy(og.dequant_mxfp4(codes[ex].numpy(), scales[ex].numpy()).astype("float32"))
            aq = oq.mxfp4_qdq(np.ascontiguousarray(ab[slots // top_k]), nthreads=cores)
            at = torch.from_numpy(aq.astype("int16")).view(torch.bfloat16).float()
            (at @ w.t()).to(torch.bfloat16)
            done_slots += len(slots)
        ex += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(2.0 * done_slots * n * k / dt / 1e12, 4), "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"{ex} of {e} experts ({done_slots} of {m * top_k} routed slots), each: C restatement of "
                      "mxfp4_qdq on the gathered tokens + dequantisation of the expert + torch fp32 matmul"}


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm on host cores (rank 0 only)
# ---------------------------------------------------------------------------


def qdq_config(workload: str) -> dict:
    wl = WORKLOADS[workload]
    return {"workload": wl["config"], "rows": wl["rows"], "cols": wl["cols"]}


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    sys.path.insert(0, str(REPO))
    from oracle import qdq as oq  # CPU restatement of the reference (test/baseline only)

    wl = WORKLOADS[args.workload]
    if args.workload in ("mxfp4_linear", "nvfp4_linear", "mxfp4_moe") or args.workload.startswith("sage3"):
        return run_reference_compute(args, wl)
    x = wl["make"]()
    cores = os.cpu_count() or 1

    def runner(rows: int):
        xb = x[:rows].view(torch.int16).numpy().view("uint16")
        if args.workload == "nvfp4_qdq":
            gs = float(global_scale_of(x)[0])
            return lambda: oq.nvfp4_qdq(xb, gs, nthreads=cores)
        if args.workload == "mxfp8_qdq":
            return lambda: oq.mxfp8_qdq(xb, nthreads=cores)
        return lambda: oq.mxfp4_qdq(xb, nthreads=cores)

    # Each step is a bounded sample of rows, sized so that warm-up + timed
    # steps take about two minutes of host time in total.
    probe_rows = min(1024, x.shape[0])
    probe = runner(probe_rows)
    probe()
    t0 = time.perf_counter()
    probe()
    per_row = (time.perf_counter() - t0) / probe_rows
    budget = 120.0 / max(1, args.steps + args.warmup)
    rows = int(max(64, min(x.shape[0], budget / max(per_row, 1e-9))))
    fn = runner(rows)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    gbs = rows * x.shape[1] * BYTES_PER_ELT / dt / 1e9
    line = {
        "impl": "reference", "metric": "QDQ HBM GB/s", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 * x.shape[0] / rows, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE shapes and distributions)",
        "config": qdq_config(args.workload),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"first {rows} of {wl['rows']} rows (x {wl['cols']} cols) per "
                                   "step; C restatement of the reference algorithm, OpenMP; rank 0 only"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def run_reference_compute(args, wl) -> None:
    """Reference arm for the GEMM / attention workloads: the reference's CPU
    emulation of the same call, each step a bounded sample (see the samplers)."""
    per_step = max(3.0, 100.0 / max(1, args.steps + args.warmup))
    if args.workload == "mxfp4_moe":
        m = args.rows or wl["rows"]
        cb = cpu_moe_sample(wl, m, budget_s=per_step * args.steps)
        metric = "FP4 MoE GEMM TFLOPS (2 x routed slots x N x K)"
        config = {"workload": wl["config"], "tokens": m, "experts": wl["E"], "top_k": wl["top_k"],
                  "N": wl["N"], "K": wl["cols"]}
        ms = 2.0 * m * wl["top_k"] * wl["N"] * wl["cols"] / (cb["value"] * 1e12) * 1e3
    elif args.workload in ("mxfp4_linear", "nvfp4_linear"):
        m = args.rows or wl["rows"]
        cb = cpu_gemm_sample(m, budget_s=per_step * args.steps)
        metric = "FP4 GEMM TFLOPS"
        config = {"workload": wl["config"], "M": m, "N": 14336, "K": 4096}
        ms = 2.0 * m * 14336 * 4096 / (cb["value"] * 1e12) * 1e3
    else:
        L = args.rows or wl["rows"]
        cb = cpu_attn_sample(wl, L, budget_s=per_step * args.steps)
        metric = "Sage3 attention TFLOPS (4*B*H*L^2*D per call)"
        config = {"workload": wl["config"], "B": wl["B"], "H": wl["H"], "L": L, "D": 128,
                  "sage3": wl["sage3"], "acc_dtype": wl["acc"]}
        ms = 4.0 * wl["B"] * wl["H"] * L * L * 128 / (cb["value"] * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": metric, "value": cb["value"], "unit": cb["unit"],
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 emulation of the FP4 path", "data": "synthetic (seeded, BASELINE shapes)",
        "config": config, "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# our arm: records
# ---------------------------------------------------------------------------


def qdq_record(ctx: Ctx, workload: str, weak: bool = False, sub: bool = False) -> dict:
    """QDQ of config 1 / 2 (or MXFP8 on config 1's input).  Strong scaling:
    rank r quantises rows row_range(M, r, N) of the one fixed tensor.  Weak
    scaling: every rank quantises a full tensor of its own (seed + rank)."""
    from vllm_qdq_plugin import _native, shard
    from vllm_qdq_plugin.qdq import mxfp4_qdq, mxfp8_qdq, nvfp4_global_scale, nvfp4_qdq, qdq_from_host

    args, wl = ctx.args, WORKLOADS[workload]
    rows = args.rows or wl["rows"]
    seed_default = {"nvfp4_qdq": 1}.get(workload, 0)
    if weak:
        x_full = wl["make"](rows=rows, seed=seed_default + ctx.rank)
        r0, r1 = 0, rows
    else:
        x_full = wl["make"](rows=rows, seed=seed_default)
        r0, r1 = ctx.share(rows)
    x_cpu = x_full[r0:r1].contiguous()
    M, K = x_cpu.shape
    # enough (x, y) pairs that each is touched again only after >= 3x the L2
    # capacity of other traffic: every timed launch reads its input from HBM
    n_pairs = max(1, -(-3 * L2_BYTES // max(1, M * K * BYTES_PER_ELT)))
    xs = [x_cpu.to(ctx.dev) for _ in range(n_pairs)]
    ys = [torch.empty_like(xs[0]) for _ in range(n_pairs)]
    lib = _native.lib()
    gs = None
    if workload == "nvfp4_qdq":
        # this rank's gs over its own rows, then one fp32 all-reduce MIN: equal to
        # 2688 / amax over the whole job's rows (strong) or over all ranks' tensors (weak)
        gs = nvfp4_global_scale(xs[0]) if M else torch.full((1,), float("inf"), device=ctx.dev)
        shard.combine_global_scale(gs)
        if not weak:
            assert torch.equal(gs.cpu(), global_scale_of(x_full)), "combined global scale != whole-tensor gs"

    def step(i, sp):
        j = i % n_pairs
        if workload == "nvfp4_qdq":
            st = lib.qdq_nvfp4(xs[j].data_ptr(), ys[j].data_ptr(), None, None, gs.data_ptr(), M, K, K, K, 0, sp)
        elif workload == "mxfp8_qdq":
            st = lib.qdq_mxfp8(xs[j].data_ptr(), ys[j].data_ptr(), None, None, M, K, K, K, 0, 32, sp)
        else:
            st = lib.qdq_mxfp4(xs[j].data_ptr(), ys[j].data_ptr(), None, None, M, K, K, K, 0, 32, sp)
        _native.check(workload, st)

    def api_call(xd):
        if workload == "nvfp4_qdq":
            return nvfp4_qdq(xd, global_scale=gs)
        return mxfp8_qdq(xd) if workload == "mxfp8_qdq" else mxfp4_qdq(xd)

    steps = args.steps
    for i in range(args.warmup):
        step(i, torch.cuda.current_stream(ctx.dev).cuda_stream)
    ms_step, clocks = timed(ctx, step, steps)
    bytes_step = M * K * BYTES_PER_ELT
    total_bytes = (rows * wl["cols"] * BYTES_PER_ELT) * (ctx.world if weak else 1)
    value = total_bytes / (ms_step * 1e-3) / 1e9

    amax = None
    if workload == "nvfp4_qdq":
        gbuf = torch.empty((1,), dtype=torch.float32, device=ctx.dev)
        wsb = torch.empty((4,), dtype=torch.int32, device=ctx.dev)

        def amax_step(i, sp):
            _native.check("qdq_nvfp4_global_scale", lib.qdq_nvfp4_global_scale(
                xs[i % n_pairs].data_ptr(), gbuf.data_ptr(), wsb.data_ptr(), M, K, K, 0, sp))

        amax_ms, _ = timed(ctx, amax_step, steps, clocks=False)
        peak, _ = measured_peak_hbm()
        amax = {"ms_per_step": round(amax_ms, 5),
                "achieved_gbs": round(M * K * 2 / (amax_ms * 1e-3) / 1e9, 1),
                "frac": round(M * K * 2 / (amax_ms * 1e-3) / 1e9 / peak, 4),
                "what": "the per-tensor global-amax pass (qdq_nvfp4_global_scale), 2 B read per element, "
                        "reported separately from the QDQ step"}

    # end to end through the public API with pinned host buffers
    x_host = x_cpu.pin_memory()
    out_host = torch.empty_like(x_cpu).pin_memory()
    host_fmt = {"nvfp4_qdq": "nvfp4", "mxfp8_qdq": "mxfp8"}.get(workload, "mxfp4")

    def e2e_step():
        qdq_from_host(x_host, host_fmt, out=out_host, device=ctx.dev, non_blocking=True,
                      global_scale=gs if host_fmt == "nvfp4" else None)

    for _ in range(2):
        e2e_step()
    ctx.barrier()
    xd = x_host.to(ctx.dev)
    local_out = api_call(xd)
    assert torch.equal(out_host.view(torch.int16), local_out.cpu().view(torch.int16)), \
        "streamed host QDQ differs from the device hook"
    e2e_steps = max(1, min(steps, 20))
    ms_e2e = timed_host(ctx, e2e_step, e2e_steps)
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9

    verified = None
    if ctx.world > 1 and not weak:
        # gather every rank's rows over NCCL (verification only) and compare with
        # one whole-tensor QDQ on rank 0
        gathered = shard.gather_rows(local_out, rows)
        if ctx.rank == 0:
            whole = api_call(x_full.to(ctx.dev))
            ok = torch.equal(gathered.view(torch.int16), whole.view(torch.int16))
            assert ok, "gathered row shards differ from a whole-tensor QDQ"
            verified = (f"{ctx.world} row shards gathered over NCCL after timing: bit-identical to one "
                        "whole-tensor QDQ")
        ctx.barrier()
    del xs, ys

    peak, peak_src = measured_peak_hbm()
    achieved = bytes_step / (ms_step * 1e-3) / 1e9
    traffic_key = {"nvfp4_qdq": "nvfp4_qdq", "mxfp4_qdq": "mxfp4_qdq", "mxfp8_qdq": "mxfp8_qdq"}[workload]
    rec = {
        "metric": "QDQ HBM GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": ctx.world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, BASELINE shapes and distributions)",
        "config": qdq_config(workload) if not args.rows else {**qdq_config(workload), "rows": rows},
        "parallelism": (f"rows x{ctx.world}: rank r owns rows row_range({rows}, r, {ctx.world}) of the one "
                        "job tensor (this rank: [%d, %d))" % (r0, r1) if not weak else
                        f"rows x{ctx.world}: every rank quantises its own [{rows}, {wl['cols']}] tensor") +
                       "; NVFP4 gs agreed by one fp32 all-reduce MIN before timing; no collective on the "
                       "data path",
        "l2": (f"{n_pairs} rotating input/output pairs of {M * K * 2 / 1e6:.0f} MB each per rank: no buffer "
               "is re-touched within 3x the 126 MB L2; steps replayed from one CUDA graph"),
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * K * 2,
                "path": (f"vllm_qdq_plugin.qdq.qdq_from_host(fmt={host_fmt!r}) on pinned host buffers: "
                         "16 MB row blocks through the C-ABI qdq_host_stream, H2D / QDQ / D2H overlapped "
                         "on three streams; bytes per rank"
                         + (f"; rank pinned to the {len(ctx.host_cpus)} CPUs NVML lists for its GPU"
                            if ctx.host_cpus else "")
                         + ("; all ranks' copies go through the one host's memory" if ctx.world > 1 else ""))},
        "gpu_launches": steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_src,
                     "traffic": ncu_traffic(traffic_key) if (M, K) == (wl["rows"], wl["cols"]) else None,
                     "algorithmic_bytes_per_launch": bytes_step,
                     "kernel": {"nvfp4_qdq": "nvfp4_vec_kernel", "mxfp8_qdq": "mxfp8_vec_kernel"}.get(
                         workload, "mxfp4_vec_kernel")},
        "clocks": clocks,
    }
    if amax:
        rec["amax"] = amax
    if verified:
        rec["verified"] = verified
    if workload == "nvfp4_qdq" and not sub:
        rec["reference_gpu"] = vllm_nvfp4_gpu(ctx, xs_local=x_cpu, gs=gs, ours_ms=ms_step)
    if ctx.world == 1 and not args.no_cpu_baseline and not sub:
        with all_host_cpus(ctx):
            rec["cpu_baseline"] = cpu_baseline(workload, x_full)
    return rec


def vllm_nvfp4_gpu(ctx: Ctx, xs_local: torch.Tensor, gs: torch.Tensor, ours_ms: float) -> dict:
    """vLLM 0.22's own GPU NVFP4 QDQ (ref_nvfp4_quant_dequant, which on a CUDA
    platform runs its Triton kernel) on this rank's rows, timed the same way,
    and compared bit for bit with this build's kernel."""
    try:
        from vllm.model_executor.layers.quantization.utils import nvfp4_emulation_utils as nv
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"vLLM import failed: {e}"}
    from vllm_qdq_plugin.qdq import nvfp4_qdq
    x = xs_local.to(ctx.dev)
    try:
        ref = nv.ref_nvfp4_quant_dequant(x, gs, 16)
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"vLLM ref_nvfp4_quant_dequant failed on the GPU: {e}"}
    same = bool(torch.equal(ref.view(torch.int16), nvfp4_qdq(x, global_scale=gs).view(torch.int16)))
    ms, _ = timed(ctx, lambda i, sp: nv.ref_nvfp4_quant_dequant(x, gs, 16), 5, graph=False, clocks=False)
    return {"impl": "vLLM 0.22 ref_nvfp4_quant_dequant on the GPU (its Triton kernel), same rows, same GPU",
            "ms_per_step": round(ms, 5), "value": round(x.numel() * BYTES_PER_ELT / (ms * 1e-3) / 1e9, 1),
            "unit": "GB/s", "speedup_of_ours": round(ms / ours_ms, 2), "bit_identical_to_ours": same}


def nvfp4_weight_of(codes: torch.Tensor, seed: int = 3) -> tuple[torch.Tensor, float]:
    """E4M3 scales per 16 for config 3's codes: exponents uniform over the
    normal E4M3 range (seeded), weight tensor scale 1/2048."""
    import numpy as np
    rng = np.random.default_rng(seed + 100)
    n, k = codes.shape[0], codes.shape[1] * 2
    exp = rng.integers(1, 16, size=(n, k // 16))
    man = np.where(exp == 15, rng.integers(0, 7, size=(n, k // 16)), rng.integers(0, 8, size=(n, k // 16)))
    return torch.from_numpy(((exp << 3) | man).astype(np.uint8)), 1.0 / 2048


def gemm_record(ctx: Ctx, m: int, sub: bool = False, marlin: bool = True, nv: bool = False) -> dict:
    """Config 3's fused linear (activation QDQ + tcgen05 FP4 GEMM): MXFP4
    (E8M0 per 32, the reference's QDQ), or with nv=True NVFP4 weights and
    activations (E4M3 per 16 + tensor scales, the VLLM_QDQ_NVFP4_ACT route).
    Strong scaling: M > 256 splits the activation rows; the decode shapes
    (M <= 256) split the 14336 output columns in 128-column blocks."""
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.gemm import (mxfp4_linear, nvfp4_linear, prepare_mxfp4_weight,
                                      prepare_nvfp4_weight)

    args = ctx.args
    wl = WORKLOADS["nvfp4_linear" if nv else "mxfp4_linear"]
    a_full, codes_full, scales_full = c3_inputs(rows=m)
    w_gs = 1.0
    if nv:
        scales_full, w_gs = nvfp4_weight_of(codes_full)
    n_full, k = codes_full.shape[0], codes_full.shape[1] * 2
    if m > 256:
        r0, r1 = ctx.share(m)
        c0, c1 = 0, n_full
        split = f"rows x{ctx.world}: rank r owns activation rows row_range({m}, r, {ctx.world})"
    else:
        b0, b1 = ctx.share(n_full // 128)
        r0, r1, c0, c1 = 0, m, 128 * b0, 128 * b1
        split = (f"output columns x{ctx.world}: rank r owns 128-column blocks unit_range({n_full // 128}, r, "
                 f"{ctx.world}) of W and C (column-parallel)")
    a_cpu = a_full[r0:r1].contiguous()
    codes, scales = codes_full[c0:c1].contiguous(), scales_full[c0:c1].contiguous()
    ml, n = a_cpu.shape[0], codes.shape[0]
    a = a_cpu.to(ctx.dev)

    def prep():
        if nv:
            return prepare_nvfp4_weight(codes.to(ctx.dev), scales.to(ctx.dev), w_gs)
        return prepare_mxfp4_weight(codes.to(ctx.dev), scales.to(ctx.dev))

    w = prep()
    # rotating weight copies: a step reads its W again only after >= 3x the
    # 126 MB L2 of other weights has streamed through
    w_bytes = w.codes.numel() + w.sf_tiled.numel()
    n_w = max(1, -(-3 * L2_BYTES // max(1, w_bytes)))
    ws_list = [w] + [prep() for _ in range(n_w - 1)]
    lib = _native.lib()
    ws_bytes = (lib.fp4_linear_nvf4_workspace_bytes if nv else lib.fp4_linear_workspace_bytes)(ml, k)
    wsp = torch.empty((ws_bytes,), dtype=torch.uint8, device=ctx.dev)
    out = torch.empty((ml, n), dtype=torch.bfloat16, device=ctx.dev)
    # MXFP4: one fused launch for M <= 64, else codes (+ scale tiling when K % 256 != 0) and the GEMM;
    # NVFP4: one fused launch for M <= 24 when N / 128 is a multiple of 4 (global amax inside),
    # else the cluster amax pass + fused launch for M <= 64; above that global amax, codes with
    # tiled scales (K % 256 == 0; else codes and a scale tiling launch), GEMM
    if nv:
        in_kernel_amax = ml <= 24 and ((n + 127) // 128) % 4 == 0
        per_call = 1 if in_kernel_amax else (2 if ml <= 64 else (3 if k % 256 == 0 else 4))
    else:
        per_call = 1 if ml <= 64 else (2 if k % 256 == 0 else 3)

    def step(i, sp):
        wi = ws_list[i % n_w]
        if nv:
            st = lib.fp4_linear_nvf4(a.data_ptr(), k, 0, None, wi.codes.data_ptr(), wi.sf_tiled.data_ptr(), w_gs,
                                     None, out.data_ptr(), ml, n, k, k // 2, n, wsp.data_ptr(), wsp.numel(), sp)
        else:
            st = lib.fp4_linear_mxf4(a.data_ptr(), k, 0, wi.codes.data_ptr(), wi.sf_tiled.data_ptr(), None,
                                     out.data_ptr(), ml, n, k, k // 2, n, wsp.data_ptr(), wsp.numel(), sp)
        _native.check("fp4_linear_nvf4" if nv else "fp4_linear_mxf4", st)

    steps = args.steps
    for i in range(args.warmup):
        step(i, torch.cuda.current_stream(ctx.dev).cuda_stream)
    ms_step, clocks = timed(ctx, step, steps)
    flop_total = 2.0 * m * n_full * k
    value = flop_total / (ms_step * 1e-3) / 1e12

    a_host = a_cpu.pin_memory()
    out_host = torch.empty((ml, n), dtype=torch.bfloat16).pin_memory()

    linear = nvfp4_linear if nv else mxfp4_linear

    def e2e_step():
        out_host.copy_(linear(a_host.to(ctx.dev, non_blocking=True), w), non_blocking=True)

    for _ in range(3):
        e2e_step()
    ms_e2e = timed_host(ctx, e2e_step, max(1, min(steps, 20)))
    e2e = flop_total / (ms_e2e * 1e-3) / 1e12

    ref = marlin_reference(ctx, a, codes, scales, w, ms_step, steps, w_gs if nv else None) if marlin else None
    peak, src = measured_peak_fp4()
    rec = {
        "metric": "FP4 GEMM TFLOPS", "value": round(value, 1), "unit": "TFLOP/s",
        "n_gpus": ctx.world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "e2m1 x e2m1 (" + ("UE4M3 scales per 16, fp32 tensor scales" if nv else "E8M0 scales") +
                 "), fp32 accumulate, bf16 out",
        "data": "synthetic (seeded, BASELINE config-3 distributions)",
        "config": {"workload": wl["config"], "M": m, "N": n_full, "K": k},
        "parallelism": split + "; no collective",
        "l2": (f"{n_w} rotating weight copies ({w_bytes / 1e6:.0f} MB each per rank): a step re-reads its W "
               "only after >= 3x the 126 MB L2; steps replayed from one CUDA graph"),
        "e2e": {"value": round(e2e, 1), "unit": "TFLOP/s", "h2d_bytes_per_step": ml * k * 2,
                "d2h_bytes_per_step": ml * n * 2,
                "path": f"vllm_qdq_plugin.gemm.{linear.__name__} on pinned host buffers (bytes per rank)"},
        "gpu_launches": steps * per_call,
        "roofline": linear_roofline(ml, n, k, ms_step, 2.0 * ml * n * k, peak, src,
                                    "nvfp4_linear" if nv else "mxfp4_linear"),
        "clocks": clocks,
    }
    if ref:
        rec["reference_gpu"] = ref
    if ctx.world == 1 and not args.no_cpu_baseline and not sub and not nv:
        with all_host_cpus(ctx):
            rec["cpu_baseline"] = cpu_gemm_sample(m)
    return rec


def marlin_reference(ctx: Ctx, a: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, w,
                     ours_ms: float, steps: int, w_gs: float | None = None) -> dict:
    """The path the fused linear replaces, on the same GPU and shapes: this
    build's activation QDQ (MXFP4: bit-exact with the reference's mxfp4_qdq;
    NVFP4, w_gs given: bit-exact with vLLM's ref_nvfp4_quant_dequant), then
    vLLM's Marlin GEMM on weights prepared by vLLM itself
    (prepare_fp4_layer_for_marlin), with the same weight rotation."""
    try:
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"vLLM import failed: {e}"}
    from vllm_qdq_plugin.gemm import mxfp4_linear, nvfp4_linear
    from vllm_qdq_plugin.qdq import mxfp4_qdq, nvfp4_qdq
    n, k = codes.shape[0], codes.shape[1] * 2
    nv = w_gs is not None
    qdq, linear = (nvfp4_qdq, nvfp4_linear) if nv else (mxfp4_qdq, mxfp4_linear)

    class _Layer(torch.nn.Module):
        pass

    def layer():
        lay = _Layer()
        lay.weight = torch.nn.Parameter(codes.to(ctx.dev), requires_grad=False)
        lay.weight_scale = torch.nn.Parameter(
            scales.to(ctx.dev).view(torch.float8_e4m3fn) if nv else scales.to(ctx.dev), requires_grad=False)
        if nv:
            lay.weight_global_scale = torch.nn.Parameter(torch.tensor(w_gs, dtype=torch.float32, device=ctx.dev),
                                                         requires_grad=False)
        lay.output_size_per_partition, lay.input_size_per_partition = n, k
        lay.params_dtype, lay.bias = torch.bfloat16, None
        mu.prepare_fp4_layer_for_marlin(lay)
        return lay

    lay0 = layer()
    w_bytes = lay0.weight.numel() * lay0.weight.element_size()
    layers = [lay0] + [layer() for _ in range(max(1, -(-3 * L2_BYTES // max(1, w_bytes))) - 1)]

    def run(i, sp, do_qdq=True):
        lay = layers[i % len(layers)]
        aq = qdq(a) if do_qdq else a_q
        return mu.apply_fp4_marlin_linear(aq, lay.weight, lay.weight_scale,
                                          lay.weight_global_scale if nv else None, lay.workspace, n, k)

    ref_out = run(0, None)
    ours_out = linear(a, w)
    same = bool(torch.equal(ref_out.view(torch.int16), ours_out.view(torch.int16)))
    rel = float((ours_out.float() - ref_out.float()).norm() / ref_out.float().norm())
    a_q = qdq(a)
    for i in range(3):
        run(i, None)
    ms_both, _ = timed(ctx, lambda i, sp: run(i, sp), steps, clocks=False)
    ms_marlin, _ = timed(ctx, lambda i, sp: run(i, sp, do_qdq=False), steps, clocks=False)
    return {"impl": (f"{qdq.__name__} (this build's kernel, bit-exact with the " +
                     ("vLLM NVFP4 emulation" if nv else "reference's") + ") + vLLM 0.22 marlin_gemm "
                     "via apply_fp4_marlin_linear, same rows/columns, same GPU, CUDA graph"),
            "ms_per_step": round(ms_both, 5), "marlin_only_ms": round(ms_marlin, 5),
            "value": round(2.0 * a.shape[0] * n * k / (ms_both * 1e-3) / 1e12, 1), "unit": "TFLOP/s (per rank)",
            "speedup_of_ours": round(ms_both / ours_ms, 2), "bit_identical_to_ours": same,
            "rel_l2_ours_vs_reference": round(rel, 6)}


def attn_record(ctx: Ctx, workload: str, steps: int | None = None, sub: bool = False,
                sdpa: bool = False) -> dict:
    """Sage3 attention.  Strong scaling over (batch, head) units: config 4's 40
    heads split across ranks; config 5's 8 batches split across ranks."""
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.sage3_attn.impl import Sage3TritonImpl

    args, wl = ctx.args, WORKLOADS[workload]
    L = args.rows or wl["rows"]
    B, H = wl["B"], wl["H"]
    if wl["B"] > 1:
        q, k, v = c5_inputs(ctx.dev, B=B, L=L, H=H)
        b0, b1 = ctx.share(B)
        q, k, v = q[b0:b1], k[b0:b1], v[b0:b1]
        split = f"batches x{ctx.world}: rank r owns batches unit_range({B}, r, {ctx.world}) (all {H} heads)"
    else:
        q, k, v = c4_inputs(ctx.dev, L=L, H=H)
        h0, h1 = ctx.share(H)
        q, k, v = (t[:, :, h0:h1] for t in (q, k, v))
        split = f"heads x{ctx.world}: rank r owns heads unit_range({H}, r, {ctx.world})"
    Bl, Hl = q.shape[0], q.shape[2]
    variant = {"mxfp4_hw": 0, "nvfp4": 1, "mxfp4": 2, "mxfp8_hw": 3}[wl["sage3"]]
    out = torch.empty(q.shape, dtype=q.dtype, device=ctx.dev)
    lib = _native.lib()
    ws = torch.empty((max(1, lib.sage3_attn_workspace_bytes(Bl, L, Hl, 128)),), dtype=torch.uint8, device=ctx.dev)
    st = [q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
          v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2)]
    strides = (ctypes.c_int64 * 12)(*st)
    sm = 1.0 / math.sqrt(128)
    acc_mode = 0 if wl["acc"] == "fp32" else 1

    def step(i, sp):
        if Bl * Hl:
            _native.check("sage3_fp4_attn", lib.sage3_fp4_attn(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), Bl, L, Hl, 128, strides, sm, variant,
                acc_mode, 0, 1, 0, ws.data_ptr(), ws.numel(), sp))

    steps = steps or max(1, min(args.steps, 10))
    for i in range(max(3, min(args.warmup, 5))):
        step(i, torch.cuda.current_stream(ctx.dev).cuda_stream)
    ms_step, clocks = timed(ctx, step, steps, graph=False)
    flop = 4.0 * B * H * L * L * 128
    value = flop / (ms_step * 1e-3) / 1e12

    impl = Sage3TritonImpl(num_heads=Hl, head_size=128, softmax_scale=sm,
                           backend_kwargs={"sage3_config": wl["sage3"], "sage3_acc_dtype": wl["acc"]})
    qh, kh, vh = (t.contiguous().cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty_like(qh).pin_memory()

    def e2e_step():
        o = impl.forward_cuda(qh.to(ctx.dev, non_blocking=True), kh.to(ctx.dev, non_blocking=True),
                              vh.to(ctx.dev, non_blocking=True))
        oh.copy_(o, non_blocking=True)

    e2e_step()
    ms_e2e = timed_host(ctx, e2e_step, 2)
    e2e = flop / (ms_e2e * 1e-3) / 1e12

    same_box = None
    if sdpa:
        same_box = sdpa_same_gpu(ctx, q, k, v, ms_step)

    fp8 = wl["sage3"] == "mxfp8_hw"
    peak, src = measured_peak_fp8() if fp8 else measured_peak_fp4()
    achieved = 4.0 * Bl * Hl * L * L * 128 / (ms_step * 1e-3) / 1e12
    at_c4 = L == 75600 and B == 1 and H == 40
    scale_fmt = "E4M3 scales per 16" if wl["sage3"] == "nvfp4" else "E8M0 scales per 32"
    rec = {
        "metric": "Sage3 attention TFLOPS (4*B*H*L^2*D per call)", "value": round(value, 1),
        "unit": "TFLOP/s", "n_gpus": ctx.world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": ("e4m3 x e4m3" if fp8 else "e2m1 x e2m1") + f" ({scale_fmt}), fp32 "
                                      "softmax/accumulate, bf16 in/out",
        "data": "synthetic (seeded, BASELINE distributions, generated on the device)",
        "config": {"workload": wl["config"], "B": B, "H": H, "L": L, "D": 128, "sage3": wl["sage3"],
                   "acc_dtype": wl["acc"]},
        "parallelism": split + "; no collective",
        "l2": "K/V code streams per head exceed L2 residency across heads; eager launches (ms-long calls)",
        "e2e": {"value": round(e2e, 1), "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * q.numel() * 2,
                "d2h_bytes_per_step": q.numel() * 2,
                "path": "Sage3TritonImpl.forward_cuda on pinned host buffers (NHD, bytes per rank)"},
        "gpu_launches": steps * 5,  # channel sums, Q pass, K pass (+delta_s), V pass, flash
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_source": src,
                     "traffic": ncu_traffic(workload) if at_c4 or not sub else None,
                     "softmax_floor_ms": round(Bl * Hl * L * L / (148 * 16 * 1.965e9) * 1e3, 2),
                     "note": "the exp2 of every score on the MUFU pipe (16/clk/SM) bounds this kernel below "
                             "the tensor peak; softmax_floor_ms is that bound for this rank's share"},
        "clocks": clocks,
    }
    if at_c4 and ctx.world == 1 and wl["sage3"] in PUBLISHED_MS:
        ref_ms = PUBLISHED_MS[wl["sage3"]]
        rec["reference_published"] = {
            "ms_per_step": ref_ms, "speedup_of_ours": round(ref_ms / ms_step, 3),
            "source": "the reference's own 1x B200 run of its Triton kernel at this shape "
                      "(scripts/bench_hw_vs_sdpa_report.md); its kernel does not run on this box"}
    if same_box:
        rec["sdpa_bf16_same_gpu"] = same_box
    if ctx.world == 1 and not args.no_cpu_baseline and not sub:
        with all_host_cpus(ctx):
            rec["cpu_baseline"] = cpu_attn_sample(wl, L)
    return rec


def sdpa_same_gpu(ctx: Ctx, q, k, v, ours_ms: float) -> dict:
    """bf16 attention on the same heads and GPU through torch's SDPA with the
    cuDNN backend (the baseline the reference's own report uses,
    scripts/bench_hw_vs_sdpa.py), else torch's default backend choice."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    qt, kt, vt = (t.permute(0, 2, 1, 3).contiguous() for t in (q, k, v))
    sdpa = torch.nn.functional.scaled_dot_product_attention
    backend = "cuDNN"
    try:
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            sdpa(qt, kt, vt)
    except RuntimeError:
        backend = "torch default"
    chosen = [SDPBackend.CUDNN_ATTENTION] if backend == "cuDNN" else list(SDPBackend)

    def run(i, sp):
        with sdpa_kernel(chosen):
            sdpa(qt, kt, vt)

    run(0, None)
    sd_ms, _ = timed(ctx, run, 2, graph=False, clocks=False)
    return {"impl": f"torch bf16 scaled_dot_product_attention ({backend} backend), same heads, same GPU",
            "ms_per_step": round(sd_ms, 3), "speedup_of_ours": round(sd_ms / ours_ms, 3)}


def moe_marlin_reference(ctx: Ctx, a, codes, scales, sidd, eidd, ntpd, twd, bs, top_k, ours_out,
                         ours_ms: float, steps: int) -> dict:
    """The path the grouped GEMM replaces, on the same GPU and routing: this
    build's mxfp4_qdq (bit-exact with the reference's) of the tokens, then
    vLLM's moe_wna16_marlin_gemm on expert weights prepared by vLLM itself
    (prepare_moe_mxfp4_layer_for_marlin), timed in a CUDA graph."""
    try:
        import vllm._custom_ops as ops
        from vllm.model_executor.layers.quantization.utils import marlin_utils_fp4 as mu
        from vllm.model_executor.layers.quantization.utils.marlin_utils import marlin_make_workspace_new
        from vllm.scalar_type import scalar_types
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"vLLM import failed: {e}"}
    from vllm_qdq_plugin.qdq import mxfp4_qdq
    e, n, kh = codes.shape
    k = kh * 2

    class _Layer(torch.nn.Module):
        pass

    lay = _Layer()
    lay.params_dtype = torch.bfloat16
    w13 = codes.to(ctx.dev)
    w13_s = scales.to(ctx.dev)
    w2 = torch.zeros((e, k, n // 4), dtype=torch.uint8, device=ctx.dev)       # the down projection is not timed
    w2_s = torch.full((e, k, n // 64), 127, dtype=torch.uint8, device=ctx.dev)
    mw13, _mw2, mw13_s, _mw2_s, _, _ = mu.prepare_moe_mxfp4_layer_for_marlin(lay, w13, w2, w13_s, w2_s, None, None)
    del w2, w2_s, _mw2, _mw2_s
    workspace = marlin_make_workspace_new(ctx.dev, 4)
    m = a.shape[0]
    out = torch.zeros((m * top_k, n), dtype=torch.bfloat16, device=ctx.dev)

    def run(i, sp):
        ops.moe_wna16_marlin_gemm(mxfp4_qdq(a), out, mw13, None, mw13_s, None, None, None, None, None, workspace,
                                  sidd, eidd, ntpd, twd, moe_block_size=bs, top_k=top_k, mul_topk_weights=True,
                                  b_q_type=scalar_types.float4_e2m1f, size_m=m, size_n=n, size_k=k, is_k_full=True,
                                  use_atomic_add=False, use_fp32_reduce=True, is_zp_float=False)

    run(0, None)
    torch.cuda.synchronize(ctx.dev)
    routed = sidd[: int(ntpd.item())]
    routed = routed[routed < m * top_k].long()
    o, r = ours_out[routed].float(), out[routed].float()
    same = bool(torch.equal(out[routed].view(torch.int16), ours_out[routed].view(torch.int16)))
    fin = torch.isfinite(o) & torch.isfinite(r)
    rel = float((o[fin] - r[fin]).norm() / r[fin].norm())
    nonfinite = {"ours": int((~torch.isfinite(o)).sum()), "reference": int((~torch.isfinite(r)).sum())}
    for i in range(2):
        run(i, None)
    ms, _ = timed(ctx, run, steps, clocks=False)
    return {"impl": "mxfp4_qdq (this build's kernel, bit-exact with the reference's) + vLLM 0.22 "
                    "moe_wna16_marlin_gemm on vLLM-prepared experts, same routing, same GPU, CUDA graph",
            "ms_per_step": round(ms, 5), "speedup_of_ours": round(ms / ours_ms, 2),
            "bit_identical_to_ours": same, "rel_l2_ours_vs_reference": round(rel, 6),
            "nonfinite_routed_values": nonfinite}


def moe_record(ctx: Ctx, sub: bool = False) -> dict:
    """Grouped MXFP4 MoE GEMM at gpt-oss-120b's w13 shape (one replica per rank)."""
    from vllm_qdq_plugin import _native
    from vllm_qdq_plugin.gemm import mxfp4_moe_linear, prepare_mxfp4_moe_weight

    args, wl = ctx.args, WORKLOADS["mxfp4_moe"]
    m = args.rows or wl["rows"]
    e, n, k, top_k = wl["E"], wl["N"], wl["cols"], wl["top_k"]
    a_cpu, codes, scales, sid, eid, ntp, topk_w, bs = moe_inputs(m, e, top_k, n, k)
    a, sidd, eidd, ntpd, twd = (t.to(ctx.dev) for t in (a_cpu, sid, eid, ntp, topk_w.reshape(-1)))
    w = prepare_mxfp4_moe_weight(codes.to(ctx.dev), scales.to(ctx.dev))
    out = torch.empty((m * top_k, n), dtype=torch.bfloat16, device=ctx.dev)
    lib = _native.lib()
    slots = int((sid < m * top_k).sum())
    ws = torch.empty((lib.fp4_moe_workspace_bytes(sidd.numel(), bs, k),), dtype=torch.uint8, device=ctx.dev)

    def step(i, sp):
        _native.check("fp4_moe_mxf4", lib.fp4_moe_mxf4(
            a.data_ptr(), k, 0, w.codes.data_ptr(), w.sf_tiled.data_ptr(), e, sidd.data_ptr(), eidd.data_ptr(),
            ntpd.data_ptr(), twd.data_ptr(), sidd.numel(), bs, top_k, 1, out.data_ptr(), n, m, n, k,
            ws.data_ptr(), ws.numel(), sp))

    for i in range(args.warmup):
        step(i, torch.cuda.current_stream(ctx.dev).cuda_stream)
    steps = max(1, min(args.steps, 200))
    ms_step, clocks = timed(ctx, step, steps)
    ref = moe_marlin_reference(ctx, a, codes, scales, sidd, eidd, ntpd, twd, bs, top_k, out, ms_step, steps)
    flop = 2.0 * slots * n * k
    value = ctx.world * flop / (ms_step * 1e-3) / 1e12
    hosts = [t.pin_memory() for t in (a_cpu, sid, eid, ntp, topk_w.reshape(-1))]
    out_host = torch.empty((m * top_k, n), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        ad, sd, ed, nd, td = (t.to(ctx.dev, non_blocking=True) for t in hosts)
        out_host.copy_(mxfp4_moe_linear(ad, w, sd, ed, nd, td, bs, top_k, True), non_blocking=True)

    for _ in range(2):
        e2e_step()
    ms_e2e = timed_host(ctx, e2e_step, 5)
    e2e = ctx.world * flop / (ms_e2e * 1e-3) / 1e12
    peak, src = measured_peak_hbm()
    fp4_peak, _ = measured_peak_fp4()
    w_bytes = w.codes.numel() + w.sf_tiled.numel()
    # algorithmic bytes: the codes and scales of every expert that owns a live
    # block, the activation rows read once, the routed output rows written once
    live = eidd[: (int(ntpd.item()) + bs - 1) // bs]
    hit = int(torch.unique(live[(live >= 0) & (live < e)]).numel())
    alg_bytes = hit * (w_bytes // e) + m * k * 2 + slots * n * 2
    achieved = alg_bytes / (ms_step * 1e-3) / 1e9
    rec = {
        "metric": "FP4 MoE GEMM TFLOPS (2 x routed slots x N x K)", "value": round(value, 1),
        "unit": "TFLOP/s", "n_gpus": ctx.world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e2m1 x e2m1 (E8M0 scales), fp32 accumulate, bf16 out",
        "data": "synthetic (seeded routing and weights)",
        "config": {"workload": wl["config"], "tokens": m, "experts": e, "top_k": top_k, "N": n, "K": k,
                   "block": bs, "routed_slots": slots},
        "parallelism": f"one replica of the layer per rank (x{ctx.world})",
        "l2": f"{w_bytes / 1e9:.2f} GB of expert weights exceed the 126 MB L2; steps replayed from one CUDA graph",
        "e2e": {"value": round(e2e, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in hosts),
                "d2h_bytes_per_step": out_host.numel() * 2,
                "path": "vllm_qdq_plugin.gemm.mxfp4_moe_linear on pinned host buffers"},
        "gpu_launches": 2 * steps,  # gather-quantise + grouped GEMM
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": src,
                     "traffic": ncu_traffic(f"mxfp4_moe_{m}"), "algorithmic_bytes": alg_bytes,
                     "experts_hit": hit, "hbm_floor_ms": round(alg_bytes / (peak * 1e9) * 1e3, 4),
                     "tensor_frac": round(flop / (ms_step * 1e-3) / 1e12 / fp4_peak, 4),
                     "kernels": "moe_gather_quant_kernel + mxf4_moe_kernel (one C-ABI call)"},
        "clocks": clocks,
    }
    rec["reference_gpu"] = ref
    if ctx.world == 1 and not args.no_cpu_baseline and not sub:
        with all_host_cpus(ctx):
            rec["cpu_baseline"] = cpu_moe_sample(wl, m)
    return rec


def linear_roofline(m: int, n: int, k: int, ms_step: float, flop: float, peak_tf: float, src: str,
                    kind: str = "mxfp4_linear") -> dict:
    """The bound of one fused linear: the FP4 tensor peak or HBM, whichever
    takes longer for its algorithmic work.  Bytes = 2MK (bf16 A) + NK/2 (W
    codes) + NK/32 (W scales; NK/16 for NVFP4) + 2MN (bf16 C); the decode
    shapes (M <= 256) are HBM-bound, config 3's M = 4096 tensor-bound."""
    nbytes = 2 * m * k + n * k // 2 + n * k // (16 if kind.startswith("nvfp4") else 32) + 2 * m * n
    hbm, hbm_src = measured_peak_hbm()
    traffic = ncu_traffic(kind if (m, n) == (4096, 14336) else f"{kind}_{m}") if n == 14336 else None
    if nbytes / (hbm * 1e9) > flop / (peak_tf * 1e12):
        achieved = nbytes / (ms_step * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "peak_source": hbm_src, "alg_bytes": nbytes,
                "traffic": traffic}
    achieved = flop / (ms_step * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tf, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tf, 4), "peak_source": src, "traffic": traffic}


def run_ours(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    # pinned staging buffers on the GPU's own NUMA node, copies from cores near its PCIe root
    from vllm_qdq_plugin import shard
    all_cpus = os.sched_getaffinity(0)
    host_cpus = shard.bind_to_gpu_cpus(local)
    ctx = Ctx(world=world, rank=rank, local=local, dev=dev, dist=dist, args=args, host_cpus=host_cpus,
              all_cpus=all_cpus)
    try:
        if args.workload is None:
            line = qdq_record(ctx, "nvfp4_qdq")
            subs = {}
            if not (args.no_sub or args.rows):
                subs["config1_mxfp4_qdq"] = qdq_record(ctx, "mxfp4_qdq", sub=True)
                subs["config3_linear_m4096"] = gemm_record(ctx, 4096, sub=True)
                subs["config3_linear_m16"] = gemm_record(ctx, 16, sub=True)
                subs["config3_nvfp4_linear_m4096"] = gemm_record(ctx, 4096, sub=True, nv=True)
                subs["config3_nvfp4_linear_m16"] = gemm_record(ctx, 16, sub=True, nv=True)
                subs["config4_sage3_mxfp4_hw"] = attn_record(ctx, "sage3_mxfp4", steps=2, sub=True, sdpa=True)
                subs["config5_sage3_nvfp4"] = attn_record(ctx, "sage3_nvfp4", steps=5, sub=True)
                subs["mxfp8_qdq_config1"] = qdq_record(ctx, "mxfp8_qdq", sub=True)
                subs["sage3_mxfp8_hw_config4_shape"] = attn_record(ctx, "sage3_mxfp8", steps=2, sub=True)
                subs["moe_gpt_oss_w13_4096_tokens"] = moe_record(ctx, sub=True)
                if world > 1:
                    subs["config2_weak_scaling"] = qdq_record(ctx, "nvfp4_qdq", weak=True, sub=True)
            line["sub_records"] = subs
        elif args.workload in ("mxfp4_linear", "nvfp4_linear"):
            line = gemm_record(ctx, args.rows or WORKLOADS[args.workload]["rows"],
                               nv=args.workload == "nvfp4_linear")
        elif args.workload == "mxfp4_moe":
            line = moe_record(ctx)
        elif args.workload.startswith("sage3"):
            line = attn_record(ctx, args.workload)
        else:
            line = qdq_record(ctx, args.workload)
        if rank == 0:
            from vllm_qdq_plugin import _native
            line["library"] = _native.library_path()
            emit(line)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


# The result line goes to the process's original stdout; everything else that
# writes to fd 1 while the bench runs (NCCL's version banner, library notices)
# is sent to stderr, so stdout carries exactly one JSON line per run.
_RESULT_FD = None


def emit(line: dict) -> None:
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, data)


def _stdout_to_stderr() -> None:
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def main() -> None:
    _stdout_to_stderr()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=None,
                    help="run one workload alone (default: config 2 headline with sub-records)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="headline only (no sub-records)")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the row count (small cases for profiling only)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        args.workload = args.workload or "nvfp4_qdq"
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
