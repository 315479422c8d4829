"""Scheduler -> worker and worker -> scheduler metadata of the vLLM connector.

Parity: reference tutti/integration/vllm/connector.py:84-178 (load/save
trackers, connector metadata) and worker_meta.py (per-rank commit counts that
the scheduler publishes only when every TP rank committed).
"""
from __future__ import annotations

from dataclasses import dataclass, field

try:  # vLLM's abstract bases when vLLM is importable; plain objects otherwise
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorMetadata as _MetaBase
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorWorkerMetadata as _WorkerMetaBase
except Exception:  # pragma: no cover - vLLM absent
    _MetaBase = object
    _WorkerMetaBase = object


@dataclass
class LoadSpec:
    """Restore ``keys`` (chunk order) into ``block_ids`` (blocks_per_chunk per key)."""

    request_id: str
    keys: list[bytes]
    block_ids: list[int]
    num_tokens: int
    is_async: bool = False


@dataclass
class SaveSpec:
    """Persist full chunks ``keys`` from ``block_ids`` after this step's forward."""

    request_id: str
    keys: list[bytes]
    block_ids: list[int]


@dataclass
class TuttiConnectorMetadata(_MetaBase):
    generation: int = 0
    loads: list[LoadSpec] = field(default_factory=list)
    saves: list[SaveSpec] = field(default_factory=list)
    step_tokens: int = 0  # tokens this step computes (the workers' step-time samples are per token)
    # requests finished since the last step whose blocks saves may still read: vLLM frees
    # their blocks now, so this step's forward must follow those saves on the device
    finished_saving: list[str] = field(default_factory=list)


@dataclass
class TuttiWorkerMetadata(_WorkerMetaBase):
    """Per-key count of ranks that committed it this step, failed loads, and the rank's measurements.

    ``read_samples``: (chunks, ms) of this rank's restores that finished (device-timed);
    ``step_samples``: (tokens, ms) of steps without a synchronous read.
    """

    committed: dict[bytes, int] = field(default_factory=dict)
    failed_loads: dict[str, int] = field(default_factory=dict)  # request id -> first failed token
    generation: int = 0  # the connector metadata this step ran with
    read_samples: list[tuple[int, float]] = field(default_factory=list)
    step_samples: list[tuple[int, float]] = field(default_factory=list)

    def aggregate(self, other: "TuttiWorkerMetadata") -> "TuttiWorkerMetadata":
        merged = dict(self.committed)
        for k, n in other.committed.items():
            merged[k] = merged.get(k, 0) + n
        failed = dict(self.failed_loads)
        for r, t in other.failed_loads.items():
            failed[r] = min(t, failed.get(r, t))
        return TuttiWorkerMetadata(merged, failed, max(self.generation, other.generation),
                                   self.read_samples + other.read_samples, self.step_samples + other.step_samples)
