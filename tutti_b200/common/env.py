"""Environment switches, read once where their defaults are needed.

| variable | effect (default) |
|---|---|
| ``TUTTI_IO_TIMING=1`` | per-command ``%globaltimer`` stamps in the io kernel (off) |
| ``TUTTI_POOL_WORKERS=<n>`` | CTAs (queue leases) one restore/store may use (the runtime option) |
| ``TUTTI_ASYNC_COMPLETION=1`` | split submit / drain launches for reads (off; read natively) |
| ``TUTTI_LOAD_MODE=sync\\|async\\|auto`` | the vLLM connector's load mode (sync) |
| ``TUTTI_CHECKPOINT_INTERVAL_S=<s>`` | object-index checkpoint cadence of the KV engine (60) |
| ``TUTTI_PRECREATE_MIN_FREE_BYTES=<n>`` | free space kept on each mount by segment-file growth |
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


def runtime_option_defaults() -> dict:
    """Runtime options that environment switches set unless the caller passes them."""
    out = {}
    if flag("TUTTI_IO_TIMING"):
        out["timing"] = True
    workers = integer("TUTTI_POOL_WORKERS")
    if workers:
        out["max_ctas_per_op"] = workers
    return out
