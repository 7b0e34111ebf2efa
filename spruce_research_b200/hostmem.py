"""Pinned host buffers placed on the GPU's own NUMA node.

A copy engine reads and writes pinned host pages over PCIe.  Pages on the
other socket cross the inter-socket link first, and with several GPUs
streaming a layer from host memory at once that link, not PCIe, sets the
pace.  Linux places a page on the node of the CPU that first touches it, and
pinning touches every page, so a buffer pinned while the process runs on the
GPU's local CPUs lands on the GPU's node.  `near(device)` binds the process to
those CPUs for the allocation and restores the previous affinity afterwards,
so nothing else (a CPU baseline using every host thread, say) is narrowed.
"""
from __future__ import annotations

import contextlib
import os

import torch


def parse_cpulist(text: str) -> set[int]:
    """CPU ids of a sysfs cpulist such as ``"0-3,8,10-11"``."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def gpu_local_cpus(device) -> set[int]:
    """The CPUs on the GPU's NUMA node that this process may run on (empty when unknown)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    props = torch.cuda.get_device_properties(idx)
    ids = [getattr(props, name, None) for name in ("pci_domain_id", "pci_bus_id", "pci_device_id")]
    if any(i is None for i in ids):
        return set()
    path = f"/sys/bus/pci/devices/{ids[0]:04x}:{ids[1]:02x}:{ids[2]:02x}.0/local_cpulist"
    try:
        with open(path) as f:
            local = parse_cpulist(f.read())
    except OSError:
        return set()
    return local & os.sched_getaffinity(0)


@contextlib.contextmanager
def near(device):
    """Run the body bound to the GPU's local CPUs; yields them (empty: unknown or not
    permitted, and the body runs unbound)."""
    cpus = gpu_local_cpus(device)
    old = os.sched_getaffinity(0)
    bound = False
    if cpus and cpus != old:
        try:
            os.sched_setaffinity(0, cpus)
            bound = True
        except OSError:  # not permitted here: allocate where the process runs
            cpus = set()
    try:
        yield cpus
    finally:
        if bound:
            os.sched_setaffinity(0, old)


def pinned_copy(t: torch.Tensor, device) -> torch.Tensor:
    """A contiguous pinned CPU copy of ``t``, placed on ``device``'s NUMA node."""
    with near(device):
        return t.contiguous().cpu().pin_memory()


def pinned_empty(shape, dtype, device) -> torch.Tensor:
    """An uninitialised pinned CPU tensor placed on ``device``'s NUMA node."""
    with near(device):
        return torch.empty(shape, dtype=dtype).pin_memory()
