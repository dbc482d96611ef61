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
