# SPDX-License-Identifier: Apache-2.0
"""Host-side partitioning for running the FP4 hot path on several GPUs.

Every kernel on this path works on independent units: QDQ and the fused
linear on rows (the GEMM's M dimension), the Sage3 attention on
(batch, head) pairs.  One process per GPU takes a contiguous range of units
and runs the single-GPU path on it; nothing crosses NVLink on the data path.
Two small exchanges sit outside it:

* NVFP4's per-tensor global scale gs = 2688 / amax(|x|) must be the same on
  every rank, or rows of the same tensor would be quantised on different
  grids.  Each rank computes gs over its own rows on the device; fp32
  division rounds monotonically, so the minimum of the per-rank values is
  exactly 2688 / (global amax).  A rank whose rows are all zero contributes
  +inf, which the minimum ignores.
* Timing takes the maximum over ranks; results are gathered only to verify
  them.

Each process can also pin itself to the host CPUs NVML lists as local to its
GPU (bind_to_gpu_cpus), so that its pinned staging buffers sit on that GPU's
NUMA node.

The reference runs one tensor per vLLM worker (src/vllm_qdq_plugin/patch.py:51-57
calls mxfp4_qdq on the worker's own activation); its vLLM tensor-parallel
ranks each quantise their own shard.  The global-scale rule follows vLLM's
NVFP4 emulation (nvfp4_emulation_utils.py:439-478), where gs is one fp32
scalar per tensor.
"""

from __future__ import annotations

import os

import torch


def unit_range(units: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of `units` owned by `rank` out of `world`.

    The first `units % world` ranks take one unit more, so the ranges tile
    [0, units) exactly with sizes differing by at most one.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if units < 0:
        raise ValueError(f"negative unit count {units}")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def row_range(rows: int, rank: int, world: int) -> tuple[int, int]:
    """Rows of a QDQ / linear input owned by `rank` (M-dimension split)."""
    return unit_range(rows, rank, world)


def head_range(batch: int, heads: int, rank: int, world: int) -> tuple[int, int]:
    """Flattened (batch * heads) pairs of an attention call owned by `rank`.

    Pair p is batch p // heads, head p % heads.
    """
    return unit_range(batch * heads, rank, world)


def combine_global_scale(gs_local: torch.Tensor, group=None) -> torch.Tensor:
    """Make the NVFP4 global scale agree across ranks, in place.

    `gs_local` is this rank's 1-element fp32 gs over its own rows (for
    example from `vllm_qdq_plugin.qdq.nvfp4_global_scale`).  After an
    all-reduce MIN it holds 2688 / amax over all ranks' rows, bit for bit
    what one GPU computes over the whole tensor.  Every rank must call this
    at the same point.
    """
    import torch.distributed as dist

    if gs_local.dtype != torch.float32 or gs_local.numel() != 1:
        raise ValueError("global scale must be a 1-element float32 tensor")
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(gs_local, op=dist.ReduceOp.MIN, group=group)
    return gs_local


def max_over_ranks(value: float, device: torch.device | str = "cpu", group=None) -> float:
    """The maximum of a per-rank scalar (a device-timed duration) over ranks."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_rows(local: torch.Tensor, rows: int, group=None) -> torch.Tensor:
    """All ranks' row blocks, concatenated in rank order (for verification).

    `local` holds this rank's `row_range(rows, rank, world)` rows.  Blocks of
    unequal size are padded to the largest for the all-gather and trimmed
    afterwards.
    """
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return local
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = row_range(rows, rank, world)
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, expected {stop - start}")
    width = -(-rows // world) if rows else 0
    padded = local.new_zeros((width,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    blocks = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(blocks, padded, group=group)
    parts = []
    for r, block in enumerate(blocks):
        s, e = row_range(rows, r, world)
        parts.append(block[: e - s])
    return torch.cat(parts, dim=0)


def gpu_cpu_affinity(device: int, nvml=None) -> list[int] | None:
    """The host CPUs NVML reports as local to CUDA device `device`.

    The device is looked up by its PCI address (CUDA and NVML may number GPUs
    differently).  Returns None when NVML is unavailable or reports nothing.
    `nvml` is the NVML module (pynvml by default); tests pass a fake.
    """
    if nvml is None:
        try:
            import pynvml as nvml
        except ImportError:
            return None
    try:
        nvml.nvmlInit()
    except Exception:
        return None
    try:
        prop = torch.cuda.get_device_properties(device)
        bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        handle = nvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = nvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 1) + 63) // 64)
        cpus = [64 * w + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1]
        return cpus or None
    except Exception:
        return None
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass


def bind_to_gpu_cpus(device: int, nvml=None) -> list[int] | None:
    """Pin this process to the CPUs local to `device` (one process per GPU).

    Pinned host buffers allocated afterwards are then first touched on the
    GPU's own NUMA node, and host copies run on cores near its PCIe root.
    Only the calling process's CPU affinity changes; no GPU setting is
    touched.  Returns the CPU list applied, or None (nothing changed) when
    NVML gives no affinity or it names no CPU this process may use.
    """
    cpus = gpu_cpu_affinity(device, nvml)
    if not cpus:
        return None
    allowed = sorted(set(cpus) & os.sched_getaffinity(0))
    if not allowed:
        return None
    os.sched_setaffinity(0, allowed)
    return allowed
