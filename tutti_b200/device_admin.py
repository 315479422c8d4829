"""Host device administration: NVMe driver binding and md RAID0 arrays.

Operator tools for a host that runs Tutti's GPU-initiated NVMe path:

* ``bind_driver(bdf, driver)``: move one PCI NVMe controller (class 0x010802)
  to ``nvme`` (the kernel's block driver) or ``snvme`` (the user-queue driver
  whose queue groups the io kernel drives). The device is unbound from its
  current driver, pinned to the new one through ``driver_override`` (only this
  device, unlike a ``new_id`` that matches every device of that vendor:device)
  and bound; the result is read back from the device's ``driver`` link.
* ``unbind_driver(driver, bdfs)``: release controllers from a driver (all of
  the devices bound to it when none are named).
* ``raid0_create(devices)``: an md RAID0 array over whole, unmounted drives
  that carry no file system and belong to no array, on the first free
  ``/dev/mdN``; ``raid0_delete(name)`` stops one. Both destroy data and refuse
  to act without ``confirm=True`` (the CLI's ``--yes``); the daemon only ever
  assembles or adopts arrays, it never creates or stops one.

Every access to the host goes through ``Host`` (sysfs, /dev, /proc and the
commands run), so the logic is tested against a fake device tree.

Parity: reference scripts/bind_nvme_device.sh (checks, unbind, bind,
verification), scripts/unbind.sh (release every snvme device),
scripts/raid0_create.sh (device safety checks, first free md name, mdadm
--create with a 64 KiB chunk) and scripts/raid0_delete.sh (mdadm --stop).
"""
from __future__ import annotations

import os
import re
import stat
import subprocess
from dataclasses import dataclass, field

BDF_RE = re.compile(r"^[0-9a-fA-F]{4}:[0-9a-fA-F]{2}:[0-9a-fA-F]{2}\.[0-7]$")
NVME_CLASS = 0x010802  # mass storage controller, non-volatile memory, NVM Express
DRIVERS = ("nvme", "snvme")
MAX_MD = 256


class AdminError(RuntimeError):
    """A check failed or the host refused an action; the message says which."""


class Host:
    """The host as the admin tools see it: file trees under roots, commands, privileges."""

    def __init__(self, sysfs: str = "/sys", dev: str = "/dev", proc: str = "/proc"):
        self.sysfs, self.dev, self.proc = sysfs, dev, proc

    def path(self, root: str, *parts: str) -> str:
        return os.path.join(root, *parts)

    def read(self, path: str) -> str:
        with open(path) as f:
            return f.read().strip()

    def write(self, path: str, value: str) -> None:
        """One write to a sysfs attribute (the kernel acts on it)."""
        with open(path, "w") as f:
            f.write(value)

    def exists(self, path: str) -> bool:
        return os.path.lexists(path)

    def listdir(self, path: str) -> list[str]:
        try:
            return sorted(os.listdir(path))
        except FileNotFoundError:
            return []

    def link_target(self, path: str) -> str | None:
        return os.path.basename(os.readlink(path)) if os.path.islink(path) else None

    def is_block_device(self, path: str) -> bool:
        try:
            return stat.S_ISBLK(os.stat(path).st_mode)
        except OSError:
            return False

    def run(self, argv: list[str]) -> tuple[int, str, str]:
        try:
            r = subprocess.run(argv, capture_output=True, text=True, timeout=120)
        except FileNotFoundError:
            return 127, "", f"{argv[0]}: not found"
        return r.returncode, r.stdout, r.stderr

    def is_root(self) -> bool:
        return os.geteuid() == 0


@dataclass
class PciDevice:
    bdf: str
    pci_class: int
    vendor: str
    device: str
    driver: str | None


@dataclass
class Report:
    """What an action did, step by step (printed by the CLI)."""

    steps: list[str] = field(default_factory=list)

    def add(self, line: str) -> None:
        self.steps.append(line)


def _need_root(host: Host) -> None:
    if not host.is_root():
        raise AdminError("must run as root")


def _device_dir(host: Host, bdf: str) -> str:
    return host.path(host.sysfs, "bus", "pci", "devices", bdf)


def _driver_dir(host: Host, driver: str) -> str:
    return host.path(host.sysfs, "bus", "pci", "drivers", driver)


def pci_device(host: Host, bdf: str) -> PciDevice:
    if not BDF_RE.match(bdf):
        raise AdminError(f"{bdf!r} is not a PCI address of the form DDDD:BB:DD.F")
    d = _device_dir(host, bdf)
    if not host.exists(d):
        raise AdminError(f"PCI device {bdf} not found")
    try:
        cls = int(host.read(os.path.join(d, "class")), 16)
        vendor = host.read(os.path.join(d, "vendor"))
        device = host.read(os.path.join(d, "device"))
    except (OSError, ValueError) as e:
        raise AdminError(f"cannot read the identity of {bdf}: {e}") from e
    return PciDevice(bdf, cls, vendor, device, host.link_target(os.path.join(d, "driver")))


def bind_driver(bdf: str, driver: str = "nvme", host: Host | None = None) -> Report:
    """Bind one NVMe controller to ``driver`` (``nvme`` or ``snvme``); verified by reading its driver link."""
    host = host or Host()
    if driver not in DRIVERS:
        raise AdminError(f"driver must be one of {DRIVERS}, got {driver!r}")
    _need_root(host)
    dev = pci_device(host, bdf)
    rep = Report()
    if dev.pci_class != NVME_CLASS:
        raise AdminError(f"{bdf} is not an NVMe controller (class 0x{dev.pci_class:06x}, want 0x{NVME_CLASS:06x})")
    rep.add(f"{bdf}: NVMe controller {dev.vendor}:{dev.device}, driver {dev.driver or 'none'}")
    ddir = _driver_dir(host, driver)
    if not host.exists(ddir):
        raise AdminError(f"the {driver} driver is not loaded (modprobe {driver})")
    devdir = _device_dir(host, bdf)
    if dev.driver == driver:
        rep.add(f"{bdf}: already bound to {driver}")
    else:
        if dev.driver is not None:
            try:
                host.write(os.path.join(_driver_dir(host, dev.driver), "unbind"), bdf)
            except OSError as e:
                raise AdminError(f"unbinding {bdf} from {dev.driver} failed: {e}") from e
            rep.add(f"{bdf}: unbound from {dev.driver}")
        try:
            host.write(os.path.join(devdir, "driver_override"), driver)
        except OSError as e:
            raise AdminError(f"setting driver_override of {bdf} failed: {e}") from e
        try:
            host.write(os.path.join(ddir, "bind"), bdf)
        except OSError as e:
            raise AdminError(f"the kernel refused to bind {bdf} to {driver}: {e} "
                             f"(check the device with lspci -k -s {bdf})") from e
        now = host.link_target(os.path.join(devdir, "driver"))
        if now != driver:
            raise AdminError(f"{bdf} is bound to {now or 'no driver'} instead of {driver}")
        rep.add(f"{bdf}: bound to {driver}")
    if driver == "nvme":
        names = [n for n in host.listdir(os.path.join(devdir, "nvme")) if n.startswith("nvme")]
        if names:
            rep.add(f"{bdf}: block controller {names[0]}")
    return rep


def bound_devices(driver: str, host: Host | None = None) -> list[str]:
    """PCI addresses bound to ``driver`` (its sysfs directory holds one link per device)."""
    host = host or Host()
    return [n for n in host.listdir(_driver_dir(host, driver)) if BDF_RE.match(n)]


def unbind_driver(driver: str = "snvme", bdfs: list[str] | None = None, host: Host | None = None) -> Report:
    """Release ``bdfs`` (default: every device bound to ``driver``) from ``driver``."""
    host = host or Host()
    if driver not in DRIVERS:
        raise AdminError(f"driver must be one of {DRIVERS}, got {driver!r}")
    _need_root(host)
    bound = bound_devices(driver, host)
    todo = bound if not bdfs else list(bdfs)
    rep = Report()
    if not todo:
        rep.add(f"no device is bound to {driver}")
        return rep
    for bdf in todo:
        if bdf not in bound:
            raise AdminError(f"{bdf} is not bound to {driver}")
        try:
            host.write(os.path.join(_driver_dir(host, driver), "unbind"), bdf)
        except OSError as e:
            raise AdminError(f"unbinding {bdf} from {driver} failed: {e}") from e
        # a later probe must not pull it straight back into the driver it left
        override = os.path.join(_device_dir(host, bdf), "driver_override")
        if host.exists(override):
            try:
                host.write(override, "\n")
            except OSError:
                pass
        rep.add(f"{bdf}: unbound from {driver}")
    return rep


def _mount_sources(host: Host) -> set[str]:
    """Devices with a mounted file system (the source field of /proc/self/mountinfo)."""
    out = set()
    try:
        text = host.read(host.path(host.proc, "self", "mountinfo"))
    except OSError:
        return out
    for line in text.splitlines():
        parts = line.split(" - ", 1)
        if len(parts) == 2:
            tail = parts[1].split()
            if len(tail) >= 2:
                out.add(tail[1])
    return out


def _check_free_drive(host: Host, device: str, mounted: set[str]) -> None:
    if not host.is_block_device(device):
        raise AdminError(f"{device} is not a block device")
    if device in mounted:
        raise AdminError(f"{device} is mounted")
    rc, out, _ = host.run(["blkid", "-p", "-o", "value", "-s", "TYPE", device])
    if rc == 0 and out.strip():
        raise AdminError(f"{device} holds a {out.strip()} file system")
    rc, out, _ = host.run(["mdadm", "--examine", device])
    if rc == 0:
        raise AdminError(f"{device} carries an md superblock (it belongs to an array)")


def next_free_md(host: Host) -> str:
    for i in range(MAX_MD):
        p = host.path(host.dev, f"md{i}")
        if not host.exists(p):
            return p
    raise AdminError(f"no free md device name below md{MAX_MD}")


def raid0_create(devices: list[str], chunk_kib: int = 64, confirm: bool = False,
                 host: Host | None = None) -> tuple[str, Report]:
    """Create an md RAID0 array over ``devices``; returns (its /dev path, report)."""
    host = host or Host()
    _need_root(host)
    if len(devices) < 2:
        raise AdminError("a RAID0 array needs at least two drives")
    if len(set(devices)) != len(devices):
        raise AdminError("a drive is named twice")
    if chunk_kib <= 0 or chunk_kib & (chunk_kib - 1) or chunk_kib < 4:
        raise AdminError("the chunk must be a power of two of at least 4 KiB")
    rc, _, _ = host.run(["mdadm", "--version"])
    if rc != 0:
        raise AdminError("mdadm is not installed")
    mounted = _mount_sources(host)
    for d in devices:
        _check_free_drive(host, d, mounted)
    md = next_free_md(host)
    rep = Report()
    rep.add(f"{md}: RAID0 over {', '.join(devices)}, {chunk_kib} KiB chunk")
    if not confirm:
        raise AdminError(f"refusing to create {md}: every byte on {', '.join(devices)} would be lost "
                         "(confirm to proceed)")
    argv = ["mdadm", "--create", md, "--level=0", f"--raid-devices={len(devices)}", *devices,
            f"--chunk={chunk_kib}K", "--run", "--verbose"]
    rc, out, err = host.run(argv)
    if rc != 0:
        raise AdminError(f"mdadm --create failed ({rc}): {(err or out).strip()[-500:]}")
    rep.add(f"{md}: created")
    return md, rep


def raid0_delete(name: str, confirm: bool = False, host: Host | None = None) -> Report:
    """Stop md array ``name`` (``md127`` or ``/dev/md127``)."""
    host = host or Host()
    _need_root(host)
    base = os.path.basename(name)
    if not re.fullmatch(r"md\d+", base):
        raise AdminError(f"{name!r} is not an md device name")
    path = host.path(host.dev, base)
    if not host.is_block_device(path):
        raise AdminError(f"{path} is not a block device")
    if path in _mount_sources(host):
        raise AdminError(f"{path} is mounted; unmount it first")
    rep = Report()
    if not confirm:
        raise AdminError(f"refusing to stop {path} without confirmation")
    rc, out, err = host.run(["mdadm", "--stop", path])
    if rc != 0:
        raise AdminError(f"mdadm --stop failed ({rc}): {(err or out).strip()[-500:]}")
    rep.add(f"{path}: stopped")
    return rep
