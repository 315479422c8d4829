"""Connector configuration -> scheduler/worker components.

``kv_connector_extra_config`` keys:
  chunk_tokens             reuse unit in tokens (multiple of the engine block size; default 256)
  namespace                key-chain namespace (default: model name + dtype)
  load_mode                sync | async | auto (default sync: layerwise restore inside the forward;
                           TUTTI_LOAD_MODE overrides)
  async_load_free_ratio    share of free blocks asynchronous loads may hold (default 0.5)
  min_retrieve_tokens      hits shorter than this are computed instead of loaded (default 0)
  max_tokens_per_load      cap on the tokens one request loads at once (default 0: no cap)
  failure_collective_timeout_s  TP failure-consensus timeout (default 30)
  lookahead_k              layers a synchronous load reads ahead of attention (default 4)
  max_inflight_saves       saves a worker keeps in flight behind the steps (default 64)
  num_layers, chunk_kv_bytes, segment_bytes   optional; checked against vLLM's KV caches
  physical_chunk_tokens    must equal chunk_tokens (one object per chunk)
  direct_transfer          true: refuse a store that moves chunks through staging buffers
  max_chunks_per_wave      accepted; a restore is one submission the io kernel pipelines
  replica_io               each GPU reads the chunks on its affine drives for every TP rank and stores
                           each rank's slice into that rank's caches over NVLink (TP > 1)
  replica_io_saves         local (default): each rank writes its own chunks; fanin: the drive-affine
                           GPUs gather every rank's blocks over NVLink and write them (with replica_io)
  kv_load_failure_policy   recompute | fail: vLLM's own kv_transfer_config field governs, applied by
                           vLLM's scheduler to the blocks the worker reports as failed
  store:
    type                   tutti | memory | a registered plugin type (tutti_nvme: Tutti's name for tutti)
    options                Tutti's nesting of root / capacity / preset (drives by device id)
    root                   namespace root (per-rank segment files under <mount>/r<rank>)
    mounts                 backing mounts, one emulated NVMe drive each (default [root])
    capacity_chunks        capacity in chunks (or capacity: "64GiB")
    segment_file_slots     slots per segment file (default 2048)
    runtime_options        options of the native runtime (leases, slots_per_lease, ...)
    segment_header_bytes   per-slot prefix bytes (a multiple of 4096; part of the on-disk layout)
    stored_format          native | fp8_block128
Placeholders ``{LOCAL_RANK}`` / ``{RANK}`` in paths are expanded per worker.
Parity: reference tutti/integration/vllm/factory.py:31-202 and
config/integration/vllm/kv_transfer.json.
"""
from __future__ import annotations

import logging
import os
import re
from dataclasses import dataclass, field

import torch

from ...common.env import text
from ...models.kv_geometry import KVGeometry

LOG = logging.getLogger("tutti_b200.vllm")

_UNITS = {"": 1, "b": 1, "kib": 1 << 10, "mib": 1 << 20, "gib": 1 << 30, "tib": 1 << 40,
          "kb": 10 ** 3, "mb": 10 ** 6, "gb": 10 ** 9, "tb": 10 ** 12}


def parse_bytes(s) -> int:
    if isinstance(s, int):
        return s
    m = re.fullmatch(r"\s*([0-9.]+)\s*([a-zA-Z]*)\s*", str(s))
    if not m or m.group(2).lower() not in _UNITS:
        raise ValueError(f"bad capacity {s!r}")
    return int(float(m.group(1)) * _UNITS[m.group(2).lower()])


def expand(path: str, rank: int, local_rank: int) -> str:
    return path.replace("{LOCAL_RANK}", str(local_rank)).replace("{RANK}", str(rank))


@dataclass
class ConnectorConfig:
    chunk_tokens: int = 256
    namespace: str = ""
    load_mode: str = "sync"
    failure_policy: str = "recompute"
    store_type: str = "tutti"
    root: str = "/tmp/tutti_kv"
    mounts: list[str] = field(default_factory=list)
    capacity_chunks: int = 0
    capacity_bytes: int = 0
    segment_file_slots: int = 2048
    runtime_options: dict = field(default_factory=dict)
    stored_format: str = "native"  # or "fp8_block128": E4M3 + 1x128 scales on disk, fused in the io kernel
    defer_writes_after_reads: bool | None = None  # None: TUTTI_DEFER_WRITES_AFTER_READS, else on
    store_options: dict = field(default_factory=dict)  # a registered third-party store type's own options
    async_load_free_ratio: float = 0.5  # async loads may hold this share of the blocks running requests leave
    preset: dict | None = None  # drives by device id (daemon config, device groups), when mounts are not given
    min_retrieve_tokens: int = 0
    max_tokens_per_load: int = 0
    failure_timeout_s: float = 30.0
    lookahead_k: int = 4  # layers restored ahead of the layer attention is waiting for
    max_inflight_saves: int = 64  # saves in flight per worker before a step waits for the oldest
    replica_io: bool = False  # drive-affine reads for every TP rank, stored over NVLink
    replica_io_saves: str = "local"  # local | fanin (drive-affine GPUs write every rank's chunks)
    expect: dict = field(default_factory=dict)  # num_layers / chunk_kv_bytes / segment_bytes given in the config
    direct_transfer: bool = False  # require the direct (paged) path
    segment_header_bytes: int = 0  # 0: the store's default

    @classmethod
    def from_extra(cls, extra: dict | None) -> "ConnectorConfig":
        extra = dict(extra or {})
        known = {"chunk_tokens", "namespace", "load_mode", "kv_load_failure_policy", "store", "async_load_free_ratio",
                 "min_retrieve_tokens", "max_tokens_per_load", "failure_collective_timeout_s", "lookahead_k",
                 "max_inflight_saves", "replica_io_saves",
                 # Tutti's keys for facts derived here from vLLM's tensors (checked, not required)
                 "num_layers", "chunk_kv_bytes", "segment_bytes", "physical_chunk_tokens",
                 "direct_transfer", "max_chunks_per_wave", "replica_io"}
        unknown = set(extra) - known
        if unknown:
            raise ValueError(f"unknown connector options: {sorted(unknown)}")
        c = cls()
        c.chunk_tokens = int(extra.get("chunk_tokens", c.chunk_tokens))
        c.namespace = str(extra.get("namespace", ""))
        # TUTTI_LOAD_MODE > load_mode in the connector config > sync
        c.load_mode = str(text("TUTTI_LOAD_MODE") or extra.get("load_mode") or c.load_mode).strip().lower()
        c.failure_policy = extra.get("kv_load_failure_policy", c.failure_policy)
        c.min_retrieve_tokens = int(extra.get("min_retrieve_tokens", 0))
        c.max_tokens_per_load = int(extra.get("max_tokens_per_load", 0))
        c.failure_timeout_s = float(extra.get("failure_collective_timeout_s", 30.0))
        c.expect = {k: int(extra[k]) for k in ("num_layers", "chunk_kv_bytes", "segment_bytes") if k in extra}
        if int(extra.get("physical_chunk_tokens", c.chunk_tokens)) != c.chunk_tokens:
            raise ValueError("physical_chunk_tokens must equal chunk_tokens here (one object per chunk)")
        c.direct_transfer = bool(extra.get("direct_transfer", False))
        if "max_chunks_per_wave" in extra and int(extra["max_chunks_per_wave"]) <= 0:
            raise ValueError("max_chunks_per_wave must be positive")
        c.replica_io = bool(extra.get("replica_io", False))
        c.replica_io_saves = str(extra.get("replica_io_saves", "local"))
        if c.replica_io_saves not in ("local", "fanin"):
            raise ValueError(f"replica_io_saves must be local or fanin, got {c.replica_io_saves!r}")
        c.lookahead_k = extra.get("lookahead_k", c.lookahead_k)
        if not isinstance(c.lookahead_k, int) or isinstance(c.lookahead_k, bool) or c.lookahead_k <= 0:
            raise ValueError(f"lookahead_k must be a positive integer, got {c.lookahead_k!r}")
        c.max_inflight_saves = extra.get("max_inflight_saves", c.max_inflight_saves)
        if not isinstance(c.max_inflight_saves, int) or isinstance(c.max_inflight_saves, bool) or \
                c.max_inflight_saves <= 0:
            raise ValueError(f"max_inflight_saves must be a positive integer, got {c.max_inflight_saves!r}")
        if c.min_retrieve_tokens < 0 or c.max_tokens_per_load < 0 or c.failure_timeout_s <= 0:
            raise ValueError("min_retrieve_tokens and max_tokens_per_load must be >= 0, the timeout > 0")
        from .load_policy import MODES, free_ratio_setting

        if c.load_mode not in MODES:
            raise ValueError(f"load_mode must be one of {MODES}, got {c.load_mode!r}")
        c.async_load_free_ratio = free_ratio_setting(extra)
        st = dict(extra.get("store", {}))
        c.store_type = st.pop("type", c.store_type)
        if c.store_type == "tutti_nvme":
            # the reference connector's schema: store {type: tutti_nvme, options: {root, capacity, preset}}
            c.store_type = "tutti"
        opts = dict(st.pop("options", {}))
        if c.store_type not in ("tutti", "memory"):
            # a store type registered by a plugin: its options are its own business
            from ...storage.registry import store_types

            if c.store_type not in store_types():
                raise ValueError(f"store.type must be one of {store_types()}, got {c.store_type!r}")
            c.store_options = {**st, **opts}
            return c
        preset = opts.pop("preset", None)
        if preset is not None:
            if not isinstance(preset, dict):
                raise ValueError("store.options.preset must be a mapping")
            # the drives a rank uses, by device id; mounts are derived per rank (storage/preset.py)
            c.preset = dict(preset)
        for k in ("root", "capacity", "capacity_chunks", "mounts", "segment_file_slots", "runtime_options",
                  "stored_format", "defer_writes_after_reads", "segment_header_bytes"):
            if k in opts:
                st.setdefault(k, opts.pop(k))
        opts.pop("io_stream", None)
        if opts:
            raise ValueError(f"unknown store options: {sorted(opts)}")
        c.root = st.pop("root", c.root)
        c.mounts = list(st.pop("mounts", []))
        c.capacity_chunks = int(st.pop("capacity_chunks", 0))
        if "capacity" in st:
            c.capacity_bytes = parse_bytes(st.pop("capacity"))
        c.segment_file_slots = int(st.pop("segment_file_slots", c.segment_file_slots))
        c.segment_header_bytes = int(st.pop("segment_header_bytes", 0))
        if c.segment_header_bytes and (c.segment_header_bytes < 4096 or c.segment_header_bytes % 4096):
            raise ValueError("segment_header_bytes must be a multiple of 4096 (at least 4096)")
        c.runtime_options = dict(st.pop("runtime_options", {}))
        c.stored_format = str(st.pop("stored_format", c.stored_format))
        dw = st.pop("defer_writes_after_reads", None)
        if dw is not None and not isinstance(dw, bool):
            raise ValueError(f"store.defer_writes_after_reads must be a bool, got {dw!r}")
        c.defer_writes_after_reads = dw
        if c.stored_format not in ("native", "fp8_block128"):
            raise ValueError("store.stored_format must be native or fp8_block128")
        if st:
            raise ValueError(f"unknown store options: {sorted(st)}")
        return c

    def capacity_for(self, geometry: KVGeometry) -> int:
        if self.capacity_chunks:
            return self.capacity_chunks
        if self.capacity_bytes:
            return max(1, self.capacity_bytes // geometry.chunk_bytes)
        return 4096


def geometry_from_layers(tensors: list[torch.Tensor], chunk_tokens: int, name: str = "vllm") -> KVGeometry:
    """KV geometry of one rank from vLLM's per-layer tensors ``[2, blocks, block_size, heads, dim]``."""
    t = tensors[0]
    if t.dim() != 5:
        raise ValueError(f"unsupported KV tensor layout {tuple(t.shape)} (expected [2, blocks, block, heads, dim])")
    planes, _, bs, heads, dim = t.shape
    return KVGeometry(name, num_layers=len(tensors), num_kv_heads=heads, head_dim=dim, block_size=bs,
                      planes=planes, dtype=t.dtype, chunk_tokens=chunk_tokens)


def store_mounts(cfg: ConnectorConfig, rank: int, local_rank: int, world: int) -> list[str]:
    """The store's mounts: explicit ``mounts``, else those of the preset's drives for this rank."""
    if cfg.mounts or not cfg.preset:
        return [expand(m, rank, local_rank) for m in cfg.mounts]
    from ...storage.preset import prepare_preset, preset_mounts

    prepared = prepare_preset(cfg.preset, rank=rank, tp_size=max(1, world))
    mounts = [expand(m, rank, local_rank) for m in preset_mounts(prepared)]
    LOG.info("[tutti] rank %d: %s preset -> drives at %s", rank, prepared["type"], mounts)
    return mounts


def make_engine(cfg: ConnectorConfig, tensors: list[torch.Tensor], rank: int, local_rank: int, world: int,
                entity: str = ""):
    """The engine of one KV entity ("" is the main KV; others get their own namespace and root).

    The store comes from the store-type registry (``cfg.store_type``); a store
    without ``get_paged`` is driven through staging buffers.
    """
    from ...engine.core import KVEngine
    from ...storage.registry import StoreContext, create_store

    g = geometry_from_layers(tensors, cfg.chunk_tokens, cfg.namespace or "vllm")
    derived = {"num_layers": g.num_layers, "chunk_kv_bytes": g.chunk_bytes, "segment_bytes": g.segment_bytes}
    for k, v in cfg.expect.items():
        if not entity and derived[k] != v:
            raise ValueError(f"{k}={v} in the connector config, but vLLM's KV caches give {derived[k]}")
    cap = cfg.capacity_for(g)
    ns = (cfg.namespace or g.fingerprint()).encode() + (b"/" + entity.encode() if entity else b"")
    device = tensors[0].device
    kind = cfg.store_type
    if kind == "tutti" and device.type != "cuda":
        kind = "memory"  # the io kernel needs the pool in HBM
    if kind == "tutti":
        options = {"root": expand(cfg.root, rank, local_rank),
                   "mounts": store_mounts(cfg, rank, local_rank, world),
                   "segment_file_slots": cfg.segment_file_slots, "runtime_options": cfg.runtime_options,
                   "stored_format": cfg.stored_format, "segment_header_bytes": cfg.segment_header_bytes}
    elif kind == "memory":
        options = {}
    else:
        options = {k: expand(v, rank, local_rank) if isinstance(v, str) else v for k, v in cfg.store_options.items()}
    ctx = StoreContext(geometry=g, capacity_chunks=cap, namespace=ns, device=device, rank=rank,
                       local_rank=local_rank, world=world, entity=entity, options=options)
    store = create_store(kind, ctx)
    media = (getattr(store, "runtime_options", None) or {}).get("emulator_media")
    if media == "memory" and os.environ.get("CUDA_MODULE_LOADING", "").upper() != "EAGER":
        # drives that DMA from this process: a kernel loaded lazily while an io kernel waits
        # on them takes a context-wide lock that also holds their copies until the io deadline
        LOG.warning("[tutti] emulated drives with memory media: start vLLM with CUDA_MODULE_LOADING=EAGER "
                    "(or warm every kernel shape up first); a lazy kernel load during a restore stalls it")
    staged = kind == "memory" or not hasattr(store, "get_paged")
    if staged and cfg.direct_transfer:
        raise ValueError(f"direct_transfer: the {kind} store on {device} moves chunks through staging buffers")
    eng = KVEngine(store, g, capacity_chunks=cap, namespace=ns, device=device, staged=staged,
                   defer_writes_after_reads=cfg.defer_writes_after_reads)
    eng.restore_from_store()
    eng.bind_layers(tensors)
    return eng
