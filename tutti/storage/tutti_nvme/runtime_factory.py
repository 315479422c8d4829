"""``tutti.storage.tutti_nvme.runtime_factory``: native runtimes from a YAML spec or a preset (tutti_b200's)."""
from tutti_b200._native import core as _core
from tutti_b200.storage.preset import normalize_preset, prepare_preset, preset_mounts  # noqa: F401
from tutti_b200.storage.preset import runtime_from_env as build_runtime_from_env  # noqa: F401
from tutti_b200.storage.preset import runtime_from_preset


def build_runtime_from_config(text: str):
    """A runtime assembled from a native runtime YAML spec (resources, resolvers, data paths, backends)."""
    return _core().make_runtime_from_config(text)


def build_runtime(preset_or_accel, mounts: list[str] | None = None, options: dict | None = None):
    """The GPU-initiated NVMe runtime: ``build_runtime(preset)`` over a preset's drives (Tutti's form), or
    ``build_runtime(accel_id, mounts, options)`` over explicit mounts (one emulated controller per mount)."""
    if isinstance(preset_or_accel, dict):
        return runtime_from_preset(preset_or_accel, int(preset_or_accel.get("gpu_id", 0) or 0), options)
    return _core().make_emulated_nvme_runtime(int(preset_or_accel), list(mounts or []), dict(options or {}))
