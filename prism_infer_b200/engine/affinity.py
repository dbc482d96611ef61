"""Host placement of a rank next to its GPU.

A serving rank feeds the block from pinned host buffers (hidden states up, outputs down). Linux
places a page on the NUMA node of the CPU that first touches it, so a buffer pinned by a thread
running on the other socket makes every copy of that rank cross the inter-socket link as well
as PCIe. ``local_to_gpu`` runs a block of host work (allocating and touching the buffers,
launching the steps) on the CPUs that NVML reports as closest to the GPU, and puts the thread's
previous CPU set back afterwards. Without NVML, or where the process may not use any of those
CPUs, it changes nothing and says so.
"""
from __future__ import annotations

import contextlib
import os


def gpu_local_cpus(device) -> set[int] | None:
    """The CPUs NVML lists as closest to ``device`` (a torch CUDA device), or None."""
    import torch
    try:
        import pynvml
    except ImportError:
        return None
    props = torch.cuda.get_device_properties(device)
    try:
        pynvml.nvmlInit()
    except pynvml.NVMLError:
        return None
    try:
        handle = None
        try:
            handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{props.uuid}")
        except pynvml.NVMLError:
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            try:
                handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except pynvml.NVMLError:
                return None
        words = ((os.cpu_count() or 64) + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
    except pynvml.NVMLError:
        return None
    finally:
        try:
            pynvml.nvmlShutdown()
        except pynvml.NVMLError:
            pass
    return {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}


@contextlib.contextmanager
def local_to_gpu(device):
    """Run the body on the CPUs nearest ``device``; yields the CPU count used (None: unchanged)."""
    try:
        before = os.sched_getaffinity(0)
    except AttributeError:
        yield None
        return
    cpus = gpu_local_cpus(device)
    use = (cpus & before) if cpus else set()
    if not use or use == before:
        yield None
        return
    os.sched_setaffinity(0, use)
    try:
        yield len(use)
    finally:
        os.sched_setaffinity(0, before)
