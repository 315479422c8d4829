"""Run a GPU's host-side work on the CPUs of that GPU's NUMA node.

A process per GPU moves KV through host memory (page-locked staging slots,
the emulated drives' in-memory images and their copy-engine DMA, the drives'
host threads). Page-locked buffers are placed on the node of the thread that
allocates them, and copy engines read them across the socket interconnect when
they sit on the other node. ``bind_to_gpu(device)`` restricts the calling
thread (and every thread it starts afterwards) to the CPUs the kernel lists as
local to the GPU's PCIe function (``/sys/bus/pci/devices/<bdf>/local_cpulist``),
intersected with the CPUs the process may already use; call it before the
runtime allocates memory or starts threads. It changes nothing outside the
process and leaves the affinity alone when the list is missing or the
intersection is empty.
"""
from __future__ import annotations

import os


def parse_cpulist(text: str) -> list[int]:
    """``"0-3,8,10-11"`` -> [0, 1, 2, 3, 8, 10, 11]."""
    out: list[int] = []
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            out.extend(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return sorted(set(out))


def gpu_pci_address(device: int) -> str:
    import torch

    p = torch.cuda.get_device_properties(device)
    return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"


def local_cpus(bdf: str, sysfs: str = "/sys") -> list[int]:
    """CPUs local to PCI function ``bdf`` (empty when the kernel does not say)."""
    path = os.path.join(sysfs, "bus", "pci", "devices", bdf.lower(), "local_cpulist")
    try:
        with open(path) as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError):
        return []


def bind_cpus(cpus: list[int]) -> list[int]:
    """Restrict the calling thread to ``cpus`` ∩ its current set; returns the set applied (empty: unchanged)."""
    allowed = sorted(set(cpus) & os.sched_getaffinity(0))
    if not allowed:
        return []
    os.sched_setaffinity(0, allowed)
    return allowed


def bind_to_gpu(device: int, sysfs: str = "/sys") -> dict:
    """Bind to GPU ``device``'s local CPUs; returns what was done (for a benchmark's record)."""
    try:
        bdf = gpu_pci_address(device)
    except Exception as e:  # noqa: BLE001 - no CUDA, no binding
        return {"bound": False, "why": f"no device properties: {e}"}
    applied = bind_cpus(local_cpus(bdf, sysfs))
    if not applied:
        return {"bound": False, "gpu": bdf, "why": "no local CPU list"}
    return {"bound": True, "gpu": bdf, "cpus": len(applied)}
