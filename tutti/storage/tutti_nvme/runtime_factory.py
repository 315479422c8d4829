"""``tutti.storage.tutti_nvme.runtime_factory``: native runtimes from a YAML spec or a preset (tutti_b200's)."""
from tutti_b200._native import core as _core
from tutti_b200.storage.preset import normalize_preset, prepare_preset, preset_mounts  # noqa: F401


def build_runtime_from_config(text: str):
    """A runtime assembled from a native runtime YAML spec (resources, resolvers, data paths, backends)."""
    return _core().make_runtime_from_config(text)


def build_runtime(accel_id: int, mounts: list[str], options: dict | None = None):
    """The GPU-initiated NVMe runtime over ``mounts`` (one emulated controller per mount)."""
    return _core().make_emulated_nvme_runtime(accel_id, mounts, dict(options or {}))
