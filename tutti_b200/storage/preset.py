"""Drive presets: which drives a rank's store uses, derived from the daemon's configuration.

A connector config may name its drives by device id only::

    store: {type: tutti_nvme, options: {root: ..., preset: {
        type: nvme-device-group,            # or local (one device) or raid0 (an md array)
        daemon_config: /etc/tutti/daemon.yaml,   # a list, or comma-separated paths
        device_groups: [[0, 1], [2, 3]]}}}  # TP ranks 0-1 use devices 0-1, ranks 2-3 devices 2-3

The daemon files are the single source of hardware facts: each device id maps
to a mount, a PCI address and a namespace. Two schemas are read: this build's
daemon (``devices: [{id, mount, pci, nsid}]``) and Tutti's (``nvmes:
[{device_id, backing_mount_path, pci_addr, namespace_id}]``); device ids must
be unique across files. Fields given explicitly in the preset win over the
daemon's. ``device_groups`` is a deployment mapping: the group count must
divide the TP size, and rank r uses group ``r // (tp / groups)``.
The derived mounts become the store's mounts (one drive per mount; a raid0
preset's members share the array's single mount).
Parity: reference tutti/storage/tutti_nvme/preset_derive.py (derive_device_fields,
daemon_config_paths), runtime_factory.py:15-80 (normalize_preset, prepare_preset,
preset_mounts) and tutti/integration/vllm/geometry.py:336-366 (apply_device_groups).
"""
from __future__ import annotations

from pathlib import Path

PRESET_TYPES = ("raid0", "nvme-device-group", "local")


def normalize_preset(preset):
    """Decimal-integer strings become ints, recursively (YAML and JSON configs disagree on quoting)."""
    if isinstance(preset, dict):
        return {k: normalize_preset(v) for k, v in preset.items()}
    if isinstance(preset, list):
        return [normalize_preset(v) for v in preset]
    if isinstance(preset, str) and preset.strip().isdigit():
        return int(preset)
    return preset


def daemon_config_paths(value) -> list[str]:
    if not value:
        return []
    if isinstance(value, (list, tuple)):
        return [str(v) for v in value if v]
    return [p.strip() for p in str(value).split(",") if p.strip()]


def load_daemon_devices(paths) -> dict[int, dict]:
    """device id -> {mount_path, pci_bdf, namespace_id} from one or more daemon files."""
    import yaml

    out: dict[int, dict] = {}
    for path in daemon_config_paths(paths):
        doc = yaml.safe_load(Path(path).read_text()) or {}
        entries = [(e.get("id"), e.get("mount"), e.get("pci"), e.get("nsid", 1)) for e in doc.get("devices") or []]
        entries += [(e.get("device_id"), e.get("backing_mount_path"), e.get("pci_addr"), e.get("namespace_id", 1))
                    for e in doc.get("nvmes") or []]
        for dev_id, mount, pci, nsid in entries:
            if dev_id is None:
                raise ValueError(f"{path}: a device entry without an id")
            dev_id = int(dev_id)
            if dev_id in out:
                raise ValueError(f"device id {dev_id} appears in more than one daemon config: {paths}")
            out[dev_id] = {"mount_path": mount, "pci_bdf": pci, "namespace_id": int(nsid)}
    return out


def apply_device_groups(preset: dict, rank: int, tp_size: int) -> dict:
    """Replace ``device_groups`` by this rank's ``devices``."""
    if "device_groups" not in preset:
        return preset
    groups = preset["device_groups"]
    if not isinstance(groups, (list, tuple)) or not groups or any(not g for g in groups):
        raise ValueError("preset.device_groups must be a non-empty list of non-empty device lists")
    if tp_size % len(groups):
        raise ValueError(f"tensor parallel size {tp_size} is not a multiple of {len(groups)} device groups")
    index = int(rank) // (tp_size // len(groups))
    if not 0 <= index < len(groups):
        raise ValueError(f"rank {rank} is outside the device groups")
    out = {k: v for k, v in preset.items() if k != "device_groups"}
    out["devices"] = [{"device_id": int(d)} for d in groups[index]]
    return out


def _derive_one(device: dict, facts: dict[int, dict]) -> dict:
    device = dict(device)
    dev_id = device.pop("device_id", None)
    if dev_id is None:
        return device  # fields given explicitly
    entry = facts.get(int(dev_id))
    if entry is None:
        raise ValueError(f"no daemon config entry for device id {dev_id}")
    for k, v in entry.items():
        device.setdefault(k, v)
    return device


def prepare_preset(preset: dict, rank: int = 0, tp_size: int = 1) -> dict:
    """Normalised preset with this rank's devices and their derived fields."""
    preset = normalize_preset(preset)
    if not isinstance(preset, dict):
        raise ValueError("preset must be a mapping")
    kind = preset.get("type", "raid0")
    if kind not in PRESET_TYPES:
        raise ValueError(f"unknown preset type {kind!r} (one of {PRESET_TYPES})")
    preset = apply_device_groups(dict(preset, type=kind), rank, tp_size)
    facts = load_daemon_devices(preset.get("daemon_config")) if preset.get("daemon_config") else {}
    if kind == "local":
        dev = dict(preset.get("device") or {})
        if "device_id" in preset:
            dev.setdefault("device_id", preset["device_id"])
        preset["devices"] = [_derive_one(dev, facts)]
    else:
        preset["devices"] = [_derive_one(d, facts) for d in preset.get("devices") or []]
    if kind == "raid0":
        mounts = preset_mounts(preset)
        if len(preset["devices"]) < 2 or not mounts or len(mounts) != 1:
            raise ValueError("a raid0 preset needs at least two members sharing one array mount")
    return preset


def preset_mounts(preset: dict) -> list[str]:
    """The distinct mounts of a prepared preset's devices, in order."""
    mounts: list[str] = []
    for d in preset.get("devices") or []:
        m = d.get("mount_path")
        if not m:
            raise ValueError(f"preset device without a mount: {d}")
        if m not in mounts:
            mounts.append(str(m))
    return mounts


def runtime_from_preset(preset: dict, accel_id: int = 0, options: dict | None = None, rank: int = 0,
                        tp_size: int = 1):
    """A GPU-initiated NVMe runtime over the preset's drives (one controller per drive mount)."""
    from .._native import core

    mounts = preset_mounts(prepare_preset(preset, rank=rank, tp_size=tp_size))
    return core().make_emulated_nvme_runtime(int(accel_id), mounts, dict(options or {}))


def runtime_from_env(accel_id: int = 0, options: dict | None = None):
    """The runtime ``TUTTI_NVME_PRESET`` describes: an inline YAML/JSON mapping or a file holding one."""
    import os

    import yaml

    raw = os.environ.get("TUTTI_NVME_PRESET", "").strip()
    if not raw:
        raise ValueError("TUTTI_NVME_PRESET is not set (an inline YAML/JSON preset or a file path)")
    preset = yaml.safe_load(Path(raw).read_text() if os.path.isfile(raw) else raw)
    if not isinstance(preset, dict):
        raise ValueError("TUTTI_NVME_PRESET must hold a mapping")
    return runtime_from_preset(preset, accel_id, options)
