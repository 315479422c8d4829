"""Store plugins by type name: the ``store.type`` of a connector config.

Two registries share one namespace of type names:

* data-plane stores (worker processes): ``register_store_type(name, factory)``
  where ``factory(ctx: StoreContext)`` returns an opened store, either staged
  (``KVStore``: register_buffer / put_batch / get_batch) or paged
  (``get_paged`` / ``put_paged`` against a registered pool, as ``TuttiKVStore``);
* scheduler-side metadata views: ``register_metadata_store_type(name,
  "module:attr")``, resolved only when a view is created, so a scheduler
  process never imports a data plane (native runtime, CUDA) through the
  registry. ``attr(options)`` returns ``None`` when nothing is on media yet,
  else an object with ``recover() -> keys``, ``contains_prefix(keys,
  all_ranks) -> int`` and ``close()``.

Built in: ``memory`` (in-process, staged), ``tutti`` and its alias
``tutti_nvme`` (segment files on NVMe through the GPU io kernel).
Parity: reference tutti/storage/registry.py:23-69 (register_store_type,
register_metadata_store_type, create_store, create_metadata_store).
"""
from __future__ import annotations

import importlib
import os
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from ..models.kv_geometry import KVGeometry


@dataclass(frozen=True)
class StoreContext:
    """What a store factory is told about the engine it serves."""

    geometry: KVGeometry
    capacity_chunks: int
    namespace: bytes
    device: torch.device
    rank: int = 0
    local_rank: int = 0
    world: int = 1
    entity: str = ""  # "" for the main KV; otherwise the entity's tag (index cache, ...)
    options: dict = field(default_factory=dict)  # the store's own options, placeholders expanded


StoreFactory = Callable[[StoreContext], Any]

_STORE_TYPES: dict[str, StoreFactory] = {}
_METADATA_STORE_TYPES: dict[str, str] = {}


def register_store_type(name: str, factory: StoreFactory) -> None:
    if not name or name in _STORE_TYPES:
        raise ValueError(f"store type {name!r} is empty or already registered")
    _STORE_TYPES[name] = factory


def register_metadata_store_type(name: str, target: str) -> None:
    if not name or name in _METADATA_STORE_TYPES:
        raise ValueError(f"metadata store type {name!r} is empty or already registered")
    if ":" not in target:
        raise ValueError("metadata store target must be 'module:attr'")
    _METADATA_STORE_TYPES[name] = target


def store_types() -> list[str]:
    return sorted(_STORE_TYPES)


def has_metadata_store(name: str) -> bool:
    return name in _METADATA_STORE_TYPES


def create_store(type_name: str, ctx: StoreContext):
    factory = _STORE_TYPES.get(type_name)
    if factory is None:
        raise ValueError(f"unknown store type {type_name!r} (registered: {store_types()})")
    return factory(ctx)


def create_metadata_store(type_name: str, options: dict):
    target = _METADATA_STORE_TYPES.get(type_name)
    if target is None:
        raise ValueError(f"store type {type_name!r} has no metadata-only view")
    module, _, attr = target.partition(":")
    obj = importlib.import_module(module)
    for part in attr.split("."):
        obj = getattr(obj, part)
    return obj(options)


# -- built-in types -------------------------------------------------------------
def _memory_store(ctx: StoreContext):
    from .memory import MemoryKVStore

    store = MemoryKVStore(ctx.geometry.chunk_bytes, capacity_chunks=ctx.capacity_chunks)
    store.open()
    return store


def _tutti_store(ctx: StoreContext):
    from .tutti_store import TuttiKVStore

    o = ctx.options
    root, mounts = o["root"], list(o.get("mounts") or [os.path.join(o["root"], "nvme0")])
    if ctx.entity:
        root = os.path.join(root, "entities", ctx.entity)
        mounts = [os.path.join(m, "entities", ctx.entity) for m in mounts]
    store = TuttiKVStore(root, ctx.geometry, capacity_chunks=ctx.capacity_chunks, mounts=mounts,
                         device=ctx.device.index, rank=ctx.rank, rank_count=ctx.world,
                         segment_file_slots=min(int(o.get("segment_file_slots", 2048)), max(16, ctx.capacity_chunks)),
                         runtime_options=dict(o.get("runtime_options") or {}), namespace=ctx.namespace,
                         stored_format=o.get("stored_format", "native"),
                         **({"segment_header_bytes": int(o["segment_header_bytes"])}
                            if o.get("segment_header_bytes") else {}))
    return store.open()


def open_tutti_metadata_view(options: dict):
    """Read-only view of a segment-file namespace (``root``, ``mounts``, ``rank``); None if absent."""
    root = options["root"]
    if not os.path.exists(os.path.join(root, "meta", "namespace")):
        return None
    from .object_layout import ObjectLayout

    mounts = list(options.get("mounts") or [os.path.join(root, "nvme0")])
    return ObjectLayout.open_view(root, mounts, rank=int(options.get("rank", 0)))


register_store_type("memory", _memory_store)
register_store_type("tutti", _tutti_store)
register_store_type("tutti_nvme", _tutti_store)
register_metadata_store_type("tutti", "tutti_b200.storage.registry:open_tutti_metadata_view")
register_metadata_store_type("tutti_nvme", "tutti_b200.storage.registry:open_tutti_metadata_view")
