"""Host placement next to the GPU (``prism_infer_b200.engine.affinity``), with NVML faked: the
block runs on the GPU's CPUs that the process may use and the previous CPU set comes back; with
no NVML answer, or no usable CPU of the GPU's, nothing changes."""
import os

import pytest

from prism_infer_b200.engine import affinity

pytestmark = pytest.mark.skipif(not hasattr(os, "sched_getaffinity"), reason="no CPU affinity")


def test_runs_on_the_gpus_cpus_and_restores(monkeypatch):
    before = os.sched_getaffinity(0)
    if len(before) < 2:
        pytest.skip("one CPU: nothing to narrow")
    near = set(sorted(before)[: len(before) // 2])
    monkeypatch.setattr(affinity, "gpu_local_cpus", lambda dev: near | {10_000})
    with affinity.local_to_gpu("cuda:0") as n:
        assert n == len(near)
        assert os.sched_getaffinity(0) == near
    assert os.sched_getaffinity(0) == before


@pytest.mark.parametrize("answer", [None, set(), {10_000}])
def test_no_usable_answer_changes_nothing(monkeypatch, answer):
    before = os.sched_getaffinity(0)
    monkeypatch.setattr(affinity, "gpu_local_cpus", lambda dev: answer)
    with affinity.local_to_gpu("cuda:0") as n:
        assert n is None
        assert os.sched_getaffinity(0) == before
    assert os.sched_getaffinity(0) == before


def test_restores_after_an_error(monkeypatch):
    before = os.sched_getaffinity(0)
    if len(before) < 2:
        pytest.skip("one CPU: nothing to narrow")
    near = {min(before)}
    monkeypatch.setattr(affinity, "gpu_local_cpus", lambda dev: near)
    with pytest.raises(RuntimeError):
        with affinity.local_to_gpu("cuda:0"):
            raise RuntimeError("step failed")
    assert os.sched_getaffinity(0) == before


class _FakeNVML:
    """The few NVML calls ``gpu_local_cpus`` makes; the UUID lookup can be made to fail."""

    class NVMLError(Exception):
        pass

    def __init__(self, uuid_ok, masks):
        self.uuid_ok, self.masks, self.calls = uuid_ok, masks, []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetHandleByUUID(self, uuid):
        self.calls.append(("uuid", uuid))
        if not self.uuid_ok:
            raise self.NVMLError("not found")
        return "h"

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        self.calls.append(("pci", bus))
        return "h"

    def nvmlDeviceGetCpuAffinity(self, handle, words):
        return self.masks[:words]


class _Props:
    uuid = "0123abcd-0000-1111-2222-333344445555"
    pci_domain_id, pci_bus_id, pci_device_id = 0, 0x1B, 0


@pytest.mark.parametrize("uuid_ok", [True, False])
def test_nvml_cpu_masks_are_decoded(monkeypatch, uuid_ok):
    import sys

    import torch
    fake = _FakeNVML(uuid_ok, [(1 << 0) | (1 << 5) | (1 << 63), 1 << 2])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda dev: _Props())
    monkeypatch.setattr(os, "cpu_count", lambda: 128)
    cpus = affinity.gpu_local_cpus("cuda:0")
    assert cpus == {0, 5, 63, 66}
    assert ("uuid", f"GPU-{_Props.uuid}") in fake.calls
    assert (("pci", "00000000:1b:00.0") in fake.calls) == (not uuid_ok)
    assert fake.calls[0] == "init" and fake.calls[-1] == "shutdown"
