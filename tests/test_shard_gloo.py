"""The multi-GPU host logic, run as two gloo ranks on the CPU.

Each rank takes its contiguous block of rows, computes the NVFP4 global scale
over its own rows (here with the CPU oracle, standing in for the device
kernel), agrees on it with the other rank, and quantises its rows.  The
gathered result must equal one quant-dequant of the whole tensor bit for bit:
rows are independent once gs agrees, which is what lets the path shard with no
collective on its data.  Also checks the max-over-ranks timing reduction.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tensor(rows: int, cols: int, zero_rows: slice | None = None) -> np.ndarray:
    """bf16 bits of N(0,1) times per-row magnitudes log-uniform in [0.01, 100]."""
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g)
    lo, hi = np.log(0.01), np.log(100.0)
    x = x * torch.exp(torch.rand(rows, 1, generator=g) * (hi - lo) + lo)
    if zero_rows is not None:
        x[zero_rows] = 0
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _rank_main(rank: int, port: int, rows: int, cols: int, zero_rows, errors) -> None:
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "vllm-qdq-plugin_b200"))
    sys.path.insert(0, str(repo))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import qdq as oq
        from vllm_qdq_plugin import shard

        x = _tensor(rows, cols, zero_rows)
        start, stop = shard.row_range(rows, rank, WORLD)
        mine = x[start:stop]
        gs = torch.tensor([oq.nvfp4_global_scale(mine) if len(mine) else float("inf")],
                          dtype=torch.float32)
        shard.combine_global_scale(gs)
        whole_gs = np.float32(oq.nvfp4_global_scale(x))
        assert np.float32(gs.item()) == whole_gs, (gs.item(), whole_gs)

        y = oq.nvfp4_qdq(mine, float(gs.item())) if len(mine) else np.zeros((0, cols), np.uint16)
        got = shard.gather_rows(torch.from_numpy(y.astype(np.int32)), rows).numpy()
        want = oq.nvfp4_qdq(x, float(whole_gs)).astype(np.int32)
        assert np.array_equal(got, want), "sharded QDQ differs from the whole-tensor QDQ"

        assert shard.max_over_ranks(1.5 + rank) == 1.5 + WORLD - 1
    except Exception as e:  # reported to the parent; every rank still reaches the barrier
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _run(rows: int, cols: int, zero_rows=None) -> None:
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, rows, cols, zero_rows, errors))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, "; ".join(msgs)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("rows", [64, 37])
def test_two_ranks_reproduce_whole_tensor_nvfp4_qdq(rows):
    _run(rows, 128)


def test_rank_with_all_zero_rows_does_not_set_the_scale():
    # rank 0's rows (the first 20 of 40) are zero: its gs is +inf
    _run(40, 64, zero_rows=slice(0, 20))


def test_unit_ranges_tile_the_units():
    from vllm_qdq_plugin import shard
    for units in (0, 1, 7, 8, 16384, 75600):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard.unit_range(units, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == units
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    assert shard.head_range(8, 24, 7, 8) == (168, 192)
    with pytest.raises(ValueError):
        shard.unit_range(10, 2, 2)
