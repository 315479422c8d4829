"""Environment switches, read once where their defaults are needed.

| variable | effect (default) |
|---|---|
| ``TUTTI_IO_TIMING=1`` | per-command ``%globaltimer`` stamps in the io kernel (off) |
| ``TUTTI_POOL_WORKERS=<n>`` | CTAs (queue leases) one restore/store may use (the runtime option) |
| ``TUTTI_ASYNC_COMPLETION=1`` | split submit / drain launches for reads (off; read natively) |
| ``TUTTI_LOAD_MODE=sync\\|async\\|auto`` | the vLLM connector's load mode (sync) |
| ``TUTTI_ASYNC_LOAD_FREE_RATIO=<r>`` | share of the blocks running requests leave that asynchronous loads may hold (0.5) |
| ``TUTTI_CHECKPOINT_INTERVAL_S=<s>`` | object-index checkpoint cadence of the KV engine (60) |
| ``TUTTI_PRECREATE_MIN_FREE_BYTES=<n>`` | free space kept on each mount by segment-file growth |
| ``TUTTI_DEFER_WRITES_AFTER_READS=0`` | writes on a stream of their own, free to overlap reads (on: writes queue behind reads) |
| ``TUTTI_PRP_MODE=dynamic\\|full_prebuild`` | validated; both name the same thing here: NVMe commands address staging slots, whose PRP lists are built once at init whatever the KV pool's size |
| ``TUTTI_REPLICA_NO_ACK=1`` | accepted; replica fan-out is push-based (the owner stores into each consumer's pool), so consumers never acknowledge and there is no ACK to skip |
| ``TUTTI_EMULATOR_MEDIA=files`` or ``memory`` | media of the emulated drives: the backing files, or a page-locked image of them that the drives DMA from into HBM staging (files) |
| ``TUTTI_DRIVE_GBPS=<x>`` | sustained transfer cap of each emulated drive in GB/s (none) |
| ``TUTTI_NVME_PRESET=<yaml or path>`` | a runtime over a preset's drives (``storage.preset.runtime_from_env``) |
| ``TUTTI_GREEN_CTX_IO_SMS``, ``TUTTI_NVTX``, ``TUTTI_METRICS_PORT``, ``TUTTI_HEALTH_INTERVAL_S``, ``TUTTI_VERBOSE`` | see their modules |
Parity: reference doc/configuration-and-performance.md:117-157 (the same names).
"""
from __future__ import annotations

import os


def flag(name: str) -> bool:
    v = os.environ.get(name, "").strip().lower()
    return v not in ("", "0", "false", "no", "off")


def integer(name: str, default: int | None = None) -> int | None:
    v = os.environ.get(name, "").strip()
    return int(v) if v else default


def number(name: str, default: float | None = None) -> float | None:
    v = os.environ.get(name, "").strip()
    return float(v) if v else default


def text(name: str, default: str | None = None) -> str | None:
    v = os.environ.get(name, "").strip()
    return v or default


PRP_MODES = ("dynamic", "full_prebuild")


def prp_mode() -> str:
    """``TUTTI_PRP_MODE`` (default ``dynamic``); anything else is a configuration error.

    Parity: reference tutti/storage/tutti_nvme/layerwise_direct.py:59-63 (same values and check).
    """
    mode = (text("TUTTI_PRP_MODE", "dynamic") or "dynamic").lower()
    if mode not in PRP_MODES:
        raise ValueError("TUTTI_PRP_MODE must be 'dynamic' or 'full_prebuild'")
    return mode


def runtime_option_defaults() -> dict:
    """Runtime options that environment switches set unless the caller passes them."""
    out = {}
    if flag("TUTTI_IO_TIMING"):
        out["timing"] = True
    workers = integer("TUTTI_POOL_WORKERS")
    if workers:
        out["max_ctas_per_op"] = workers
    media = text("TUTTI_EMULATOR_MEDIA")
    if media:
        if media not in ("files", "memory"):
            raise ValueError("TUTTI_EMULATOR_MEDIA must be 'files' or 'memory'")
        out["emulator_media"] = media
    gbps = number("TUTTI_DRIVE_GBPS")
    if gbps:
        out["drive_gbps"] = gbps
    if flag("TUTTI_DIRECT_READS"):
        out["direct_reads"] = True
    return out
