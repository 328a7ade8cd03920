"""CPU: bench.py's clock summary and CPU-set handling (no GPU, no nvidia-smi)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import bench  # noqa: E402

ACTIVE = ["0", "1965", "1965", "500", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"]
CAPPED = ["0", "1900", "1965", "900", "0x4", "Not Active", "Not Active", "Not Active", "Active"]


def _sampler(samples):
    c = bench.ClockSampler(0)
    c.samples = list(samples)
    return c


def test_clock_summary_inside_region():
    c = _sampler([(1.0, ACTIVE), (1.1, CAPPED), (2.0, ACTIVE)])
    got = c.summary(1.05, 1.15)
    assert got["samples_inside_timed_region"] == 1
    assert got["sm_mhz"] == 1900.0 and got["reasons"] == ["sw_power_cap"]


def test_clock_summary_short_region_uses_neighbours():
    # a region shorter than the sampling period: the samples within 0.25 s of it count
    c = _sampler([(1.0, ACTIVE), (1.2, CAPPED), (5.0, CAPPED)])
    got = c.summary(1.1, 1.1001)
    assert got["samples_inside_timed_region"] == 0
    assert got["samples"] == 2 and got["sm_mhz"] == (1965.0 + 1900.0) / 2


def test_clock_summary_without_samples():
    assert _sampler([]).summary(0.0, 1.0) is None


def test_all_host_cpus_restores_the_binding():
    start = os.sched_getaffinity(0)
    one = [sorted(start)[0]]
    ctx = bench.Ctx(world=1, rank=0, local=0, dev=None, dist=None, args=None, host_cpus=one, all_cpus=start)
    os.sched_setaffinity(0, one)
    try:
        with bench.all_host_cpus(ctx):
            assert os.sched_getaffinity(0) == start
        assert os.sched_getaffinity(0) == set(one)
    finally:
        os.sched_setaffinity(0, start)


def test_all_host_cpus_without_binding_is_a_no_op():
    start = os.sched_getaffinity(0)
    ctx = bench.Ctx(world=1, rank=0, local=0, dev=None, dist=None, args=None)
    with bench.all_host_cpus(ctx):
        assert os.sched_getaffinity(0) == start
