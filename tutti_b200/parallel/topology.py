"""PCIe topology: which GPU each NVMe drive sits closest to.

A drive-affine restore reads each drive from the GPU behind the same PCIe
switch. The switch tree is in sysfs: ``/sys/bus/pci/devices/<bdf>`` links to a
path through every bridge above the device (``.../pci0000:00/0000:00:01.0/
0000:01:00.0/0000:02:08.0/0000:05:00.0``). Two devices under the same switch
share a longer prefix of bridges than devices on different root ports; the
affine GPU of a drive is the GPU with the longest shared prefix (the lowest
GPU index wins a tie).

``discover`` lists NVMe controllers (PCI class 0x0108xx) and NVIDIA GPUs
(vendor 0x10de, class 0x03xxxx); ``affine_gpus`` turns a drive list into the
``affine_gpus`` argument of the fan-out restore/store.
Parity: reference scripts/pci_topology_check.sh (GPU <-> NVMe switch
affinity) and doc/configuration-and-performance.md (DEVICE_GROUPS).
"""
from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class PciDevice:
    bdf: str
    path: tuple[str, ...]  # bridges from the root complex down to the device itself
    kind: str              # "nvme" | "gpu"


def _read(path: str) -> str:
    try:
        with open(path) as f:
            return f.read().strip()
    except OSError:
        return ""


def pci_path(sysfs_root: str, bdf: str) -> tuple[str, ...]:
    """The chain of PCI addresses from the root port to ``bdf`` (from the sysfs device link)."""
    real = os.path.realpath(os.path.join(sysfs_root, "bus", "pci", "devices", bdf))
    parts = [p for p in real.split(os.sep) if p.count(":") == 2 and "." in p]
    return tuple(parts)


def discover(sysfs_root: str = "/sys") -> list[PciDevice]:
    base = os.path.join(sysfs_root, "bus", "pci", "devices")
    out = []
    try:
        names = sorted(os.listdir(base))
    except OSError:
        return out
    for bdf in names:
        cls = _read(os.path.join(base, bdf, "class")).lower()
        vendor = _read(os.path.join(base, bdf, "vendor")).lower()
        if cls.startswith("0x0108"):
            out.append(PciDevice(bdf, pci_path(sysfs_root, bdf), "nvme"))
        elif vendor == "0x10de" and cls.startswith("0x03"):
            out.append(PciDevice(bdf, pci_path(sysfs_root, bdf), "gpu"))
    return out


def _shared(a: tuple[str, ...], b: tuple[str, ...]) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def affinity(drives: list[PciDevice], gpus: list[PciDevice]) -> list[int]:
    """For each drive, the index (into ``gpus``) of the GPU sharing the most PCIe bridges with it."""
    if not gpus:
        raise ValueError("no GPUs to map drives to")
    out = []
    for d in drives:
        best = max(range(len(gpus)), key=lambda i: (_shared(d.path[:-1], gpus[i].path[:-1]), -i))
        out.append(best)
    return out


def affine_gpus(sysfs_root: str = "/sys") -> list[int]:
    """Drive-affine GPU index for each NVMe controller, in PCI address order ([] without drives)."""
    devs = discover(sysfs_root)
    drives = [d for d in devs if d.kind == "nvme"]
    gpus = [d for d in devs if d.kind == "gpu"]
    return affinity(drives, gpus) if drives and gpus else []
