"""Several KV entities per attention layer (e.g. the main KV plus an index cache).

Models such as DeepSeek-V3.2 and MiniMax-M3 keep a second cache beside the
attention KV: a per-token fp8 index cache with its own page size. Each entity
gets its own engine and store namespace (its own segment-file geometry); the
same chunk keys and block ids address both, a chunk counts as resident only
when every entity holds it, and a layer is ready when every entity's copy of
that layer is.
Parity: reference tutti/integration/vllm/minimax.py (main + index cache
callbacks per attention layer) and tutti/storage/tutti_nvme/layerwise_direct.py
(per-entity page geometry).
"""
from __future__ import annotations

from typing import Sequence

from .completion import AggregateCompletion, LoadGateError


class _AllIndex:
    def __init__(self, engines):
        self._engines = engines

    def is_resident(self, key: bytes) -> bool:
        return all(e.index.is_resident(key) for e in self._engines)


class _MultiPlan:
    """Layerwise read plans of every entity; ``wait_layer`` takes the connector's layer ordinal."""

    def __init__(self, plans, layer_map: Sequence[tuple[int, int]]):
        self._plans = plans
        self._layer_map = list(layer_map)

    def wait_layer(self, layer: int) -> None:
        ent, local = self._layer_map[layer]
        self._plans[ent].wait_layer(local)

    def finish(self) -> None:
        failed, first = set(), None
        for p in self._plans:
            try:
                p.finish() if hasattr(p, "finish") else p.wait()
            except Exception as e:  # noqa: BLE001 - merged below
                first = first or e
                failed.update(getattr(e, "failed_chunks", ()))
        if first is not None:
            raise LoadGateError(f"restore failed: {first}", failed or getattr(first, "failed_chunks", ()))

    def abort(self) -> None:
        for p in self._plans:
            if hasattr(p, "abort"):
                p.abort()

    def read_ms(self) -> float | None:
        """The slowest entity's read time (entities read in parallel), once every plan knows its own."""
        times = [p.read_ms() if hasattr(p, "read_ms") else None for p in self._plans]
        return None if any(t is None for t in times) else max(times)


class _Stores:
    def __init__(self, engines):
        self._engines = engines
        self.main = engines[0].store

    def __getattr__(self, name):
        return getattr(self.main, name)

    def close(self) -> None:
        for e in self._engines:
            if hasattr(e.store, "close"):
                e.store.close()


class EntityEngines:
    """One engine per KV entity behind the single-engine interface the connector's worker uses."""

    def __init__(self, engines, layer_map: Sequence[tuple[int, int]], names: Sequence[str] = ()):
        if not engines:
            raise ValueError("no entities")
        self.engines = list(engines)
        self.layer_map = list(layer_map)
        self.names = list(names)
        self.index = _AllIndex(self.engines)
        self.store = _Stores(self.engines)

    @property
    def staged(self) -> bool:
        return all(e.staged for e in self.engines)

    def load(self, keys, block_table):
        return AggregateCompletion([e.load(keys, block_table) for e in self.engines])

    def start_read_plan(self, keys, block_table, window: int = 4):
        return _MultiPlan([e.start_read_plan(keys, block_table, window=window) for e in self.engines], self.layer_map)

    def store_chunks(self, keys, block_table, *, after=None):
        parts = [e.store_chunks(keys, block_table, after=after) for e in self.engines]
        parts = [p for p in parts if p is not None]
        return AggregateCompletion(parts) if parts else None

    def wait_idle(self) -> None:
        for e in self.engines:
            e.wait_idle()
