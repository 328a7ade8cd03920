"""CPU: binding a rank to the host CPUs local to its GPU (vllm_qdq_plugin.shard).

NVML is replaced by a fake; the CPU list comes from its affinity bitmask, the
device is found by PCI address, and the process affinity is only narrowed to
CPUs it may already use.
"""

from __future__ import annotations

import os
import types

import pytest

from vllm_qdq_plugin import shard


class FakeNvml:
    def __init__(self, words, fail_init=False):
        self.words = words
        self.fail_init = fail_init
        self.bus = None
        self.shutdown = 0

    def nvmlInit(self):
        if self.fail_init:
            raise RuntimeError("no driver")

    def nvmlShutdown(self):
        self.shutdown += 1

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        self.bus = bus
        return "handle"

    def nvmlDeviceGetCpuAffinity(self, handle, n_words):
        assert handle == "handle" and n_words >= 1
        return self.words


@pytest.fixture
def fake_props(monkeypatch):
    props = types.SimpleNamespace(pci_domain_id=0, pci_bus_id=0x1B, pci_device_id=0)
    monkeypatch.setattr(shard.torch.cuda, "get_device_properties", lambda dev: props)
    return props


def test_affinity_bitmask_to_cpu_list(fake_props):
    nvml = FakeNvml([0b1011, 1 << 1])
    assert shard.gpu_cpu_affinity(0, nvml) == [0, 1, 3, 65]
    assert nvml.bus == "00000000:1b:00.0"
    assert nvml.shutdown == 1


def test_affinity_unavailable(fake_props):
    assert shard.gpu_cpu_affinity(0, FakeNvml([0], fail_init=True)) is None
    assert shard.gpu_cpu_affinity(0, FakeNvml([0])) is None


def test_bind_narrows_to_allowed_cpus(fake_props, monkeypatch):
    allowed = sorted(os.sched_getaffinity(0))
    mask = 0
    for c in allowed[:2] + [4095]:  # CPU 4095 is not one this process may use
        if c < 64:
            mask |= 1 << c
    words = [mask] + [0] * 62 + [1 << 63]
    applied = {}
    monkeypatch.setattr(shard.os, "sched_setaffinity", lambda pid, cpus: applied.setdefault("cpus", list(cpus)))
    got = shard.bind_to_gpu_cpus(0, FakeNvml(words))
    want = [c for c in allowed[:2] if c < 64]
    if want:
        assert got == want and applied["cpus"] == want
    else:
        assert got is None and not applied


def test_bind_without_nvml_changes_nothing(fake_props, monkeypatch):
    monkeypatch.setattr(shard.os, "sched_setaffinity", lambda pid, cpus: pytest.fail("affinity changed"))
    assert shard.bind_to_gpu_cpus(0, FakeNvml([0], fail_init=True)) is None
