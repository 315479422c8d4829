"""KVEngine: the semantic index plus the execution of restores and stores.

Planning state lives in the ``ChunkIndex`` (residency, pins, pending writes,
LRU eviction). Execution goes through a store:

* direct (``TuttiKVStore`` with the engine's paged pool registered once): a
  restore is one ``get_paged`` per layer whose fused io kernel scatters into
  the pool's blocks; a store is one ``put_paged`` whose io kernel gathers them;
* staged (any ``KVStore``, e.g. ``MemoryKVStore``): chunk bytes move through a
  staging buffer with the bulk-copy gather/scatter kernels.

Layerwise restores (``start_read_plan``): a feeder thread submits layer
l's restore on a high-priority IO stream and records an event per layer;
``wait_layer(l)`` makes the *current* stream wait on that event on the
device, so attention of layer l starts as soon as its KV is in HBM while
layers l+1.. are still being read. Writes are queued behind a compute event
and settled (index confirm, object commit) when they complete.

Write ordering (``defer_writes_after_reads``, default on): writes share the IO
stream with reads, so a write's io kernel starts only after every read
submitted before it; mixed read/write traffic on one drive slows both. Off,
writes get their own stream and may overlap reads (useful when writes would
otherwise starve behind a continuous read stream); ``wait_write_stream_event``
still lets a caller order one write batch after a given event.
Parity: reference tutti/engine/core.py:53-2842 (_ReadPlan, _AsyncReadPlan,
_DirectAllLayerReadPlan with its feeder thread, _QueuedWrite, KVEngine).
"""
from __future__ import annotations

import collections
import logging
import threading
import time
from typing import Sequence

import numpy as np
import torch

from ..common.env import flag, number, text
from ..common.observability import nvtx_range
from ..index.chunk_index import ChunkIndex, StorePlan
from ..models.kv_geometry import KVGeometry
from ..parallel.green_context import configured_io_sms, io_stream_on_sms
from .completion import LoadGateError, PostCompletion, TimedCompletion
from .staging import StagingBuffer

LOG = logging.getLogger("tutti_b200.engine")
FEEDER_WAIT_S = 120.0


def resolve_defer_writes(value: bool | None) -> bool:
    """Explicit option, else ``TUTTI_DEFER_WRITES_AFTER_READS`` ("0" turns it off), else on.

    Parity: reference tutti/storage/tutti_nvme/store.py:1711-1727 (same precedence and default).
    """
    if value is None:
        env = text("TUTTI_DEFER_WRITES_AFTER_READS")
        return True if env is None else env != "0"
    if not isinstance(value, bool):
        raise ValueError(f"defer_writes_after_reads must be a bool, got {value!r}")
    return value


class LayerwiseReadPlan:
    """Per-layer restore of ``keys`` into ``block_table`` rows, fed by a thread."""

    def __init__(self, engine: "KVEngine", keys: Sequence[bytes], block_table: np.ndarray,
                 layers: Sequence[int], io_stream: torch.cuda.Stream, window: int = 4):
        self.engine = engine
        self.keys = list(keys)
        self.block_table = block_table
        self.layers = list(layers)
        self.io_stream = io_stream
        self.window = max(1, window)
        self._events: dict[int, torch.cuda.Event] = {}
        self._comp_of: dict[int, object] = {}
        self._comps: list = []
        self._cv = threading.Condition()
        self._error: BaseException | None = None
        self._closed = False
        self.t_submit0 = time.perf_counter()
        self.read_done_s: float | None = None
        # read time: the IO stream's events around all layers; with split completion the
        # last drain runs on the consumer stream, so the end is recorded there instead
        self._ev_start: torch.cuda.Event | None = None
        self._ev_end_consumer: torch.cuda.Event | None = None
        self._thread = threading.Thread(target=self._feed, name="tutti-feeder", daemon=True)
        self._thread.start()

    def _feed(self) -> None:
        store = self.engine.store
        dev = self.engine.device
        try:
            torch.cuda.set_device(dev)
            start = torch.cuda.Event(enable_timing=True)
            start.record(self.io_stream)
            self._ev_start = start
            for li, layer in enumerate(self.layers):
                if self._closed:
                    break
                # at most `window` layers in flight (queue leases are shared)
                if li >= self.window:
                    self._comps[li - self.window].wait()
                with nvtx_range(f"tutti.layer_load|layer={layer}|chunks={len(self.keys)}"):
                    comp = store.get_paged(self.keys, self.block_table, layers=[layer], stream=self.io_stream)
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(self.io_stream)
                with self._cv:
                    self._comps.append(comp)
                    self._comp_of[layer] = comp
                    self._events[layer] = ev
                    self._cv.notify_all()
        except BaseException as e:  # noqa: BLE001 - surfaced by wait_layer / finish
            with self._cv:
                self._error = e
                self._cv.notify_all()

    def wait_layer(self, layer: int) -> None:
        """Order the current stream after layer ``layer``'s restore (device-side wait)."""
        deadline = time.monotonic() + FEEDER_WAIT_S
        with self._cv:
            while layer not in self._events and self._error is None:
                left = deadline - time.monotonic()
                if left <= 0:
                    raise LoadGateError(f"feeder did not submit layer {layer} within {FEEDER_WAIT_S}s")
                self._cv.wait(timeout=left)
            if layer not in self._events:
                raise LoadGateError(f"restore of layer {layer} failed: {self._error}")
            ev = self._events[layer]
            comp = self._comp_of.get(layer)
        with nvtx_range(f"tutti.layer_wait|layer={layer}"):
            if comp is not None and self.engine.host_gated_layer_waits:
                try:
                    comp.wait()  # the host waits; the stream then waits on a finished event
                except Exception as e:  # noqa: BLE001 - surfaced like a feeder failure
                    raise LoadGateError(f"restore of layer {layer} failed: {e}") from e
                torch.cuda.current_stream().wait_event(ev)
            elif comp is not None and hasattr(comp, "enqueue_wait"):
                # device-side wait on the restore itself; with split completion this
                # launches the drain here, on the consumer's stream
                comp.enqueue_wait(torch.cuda.current_stream())
            else:
                torch.cuda.current_stream().wait_event(ev)
            if layer == self.layers[-1] and self.engine.split_completion:
                end = torch.cuda.Event(enable_timing=True)
                end.record(torch.cuda.current_stream())
                self._ev_end_consumer = end

    def finish(self) -> None:
        """Host-wait for every layer; raises LoadGateError listing the failed chunks."""
        self._thread.join(timeout=FEEDER_WAIT_S)
        failed: set[int] = set()
        err = self._error
        for comp in self._comps:
            try:
                comp.wait()
            except Exception as e:  # noqa: BLE001
                err = err or e
                per_layer = len(self.keys) * self.engine.geometry.blocks_per_chunk * self.engine.geometry.planes
                for i in getattr(e, "failed", []):
                    failed.add((i % per_layer) // (self.engine.geometry.blocks_per_chunk * self.engine.geometry.planes))
        self.read_done_s = time.perf_counter() - self.t_submit0
        if err is not None:
            raise LoadGateError(f"restore failed: {err}", failed or range(len(self.keys)))

    def abort(self) -> None:
        self._closed = True
        try:
            self.finish()
        except LoadGateError:
            pass

    def read_ms(self) -> float | None:
        """Device time from the first layer's submission to the last layer's data, once known."""
        start = self._ev_start
        end = self._ev_end_consumer if self.engine.split_completion else self._events.get(self.layers[-1])
        if start is None or end is None or not end.query():
            return None
        return float(start.elapsed_time(end))


class _WholeRestorePlan:
    """The plan interface over one finished restore (a host-memory pool has no streams to overlap)."""

    def __init__(self, comp):
        self._comp = comp

    def wait_layer(self, layer: int) -> None:
        return None

    def finish(self) -> None:
        self._comp.wait()

    def abort(self) -> None:
        pass

    def read_ms(self) -> float | None:
        return self._comp.read_ms()


class KVEngine:
    def __init__(self, store, geometry: KVGeometry, *, capacity_chunks: int | None = None,
                 namespace: bytes = b"", device: int | torch.device = 0, staged: bool | None = None,
                 io_priority: int = -1, checkpoint_interval_s: float | None = None,
                 defer_writes_after_reads: bool | None = None):
        self.store = store
        self.geometry = geometry
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        cap = capacity_chunks or getattr(store, "capacity_chunks", 1 << 20)
        self.index = ChunkIndex(cap, geometry.chunk_tokens, namespace)
        self.staged = (not hasattr(store, "get_paged")) if staged is None else staged
        self.pool: torch.Tensor | None = None
        self._io_stream: torch.cuda.Stream | None = None
        self._io_priority = io_priority
        self._write_stream: torch.cuda.Stream | None = None
        self.defer_writes_after_reads = resolve_defer_writes(defer_writes_after_reads)
        self._writes: collections.deque = collections.deque()
        self._staging_bufs: dict[str, StagingBuffer] = {}  # staged stores: one reused buffer per direction
        self._checkpoint_interval = (checkpoint_interval_s if checkpoint_interval_s is not None
                                     else number("TUTTI_CHECKPOINT_INTERVAL_S", 60.0))
        self._last_checkpoint = time.monotonic()
        self.stats = collections.Counter()

    # -- index forwarding ---------------------------------------------------
    def hash_keys(self, tokens: Sequence[int], **kw):
        return self.index.hash_keys(tokens, **kw)

    def lookup_prefix(self, tokens: Sequence[int]) -> int:
        return self.index.lookup_prefix(tokens)

    def lookup_prefix_keys(self, keys: Sequence[bytes]) -> int:
        return self.index.lookup_prefix_keys(keys)

    def pin(self, keys) -> None:
        self.index.pin(keys)

    def unpin(self, keys) -> None:
        self.index.unpin(keys)

    def begin_step(self, max_pending_age: int = 64) -> int:
        """Advance the index epoch; reclaim reservations no rank ever settled."""
        self.index.advance_epoch()
        stale = self.index.reclaim_stale_pending(max_pending_age)
        if stale:
            LOG.warning("reclaimed %d stale pending reservation(s)", len(stale))
        self.poll_writes()
        return self.index.epoch

    def restore_from_store(self) -> int:
        """Cold start: publish chunks the store already holds."""
        if hasattr(self.store, "scan"):
            keys = list(self.store.scan())
            self.index.restore(keys)
            return len(keys)
        return 0

    # -- binding --------------------------------------------------------------
    @property
    def io_stream(self) -> torch.cuda.Stream:
        if self._io_stream is None:
            sms = configured_io_sms()
            if sms:
                # io kernels confined to a green-context SM partition (TUTTI_GREEN_CTX_IO_SMS)
                dev = self.device.index if isinstance(self.device, torch.device) else int(self.device)
                self._io_stream = io_stream_on_sms(sms, dev or 0)
            else:
                self._io_stream = torch.cuda.Stream(device=self.device, priority=self._io_priority)
        return self._io_stream

    @property
    def write_stream(self) -> torch.cuda.Stream:
        """The stream writes are submitted on: the IO stream (writes after reads) or a stream of their own."""
        if self.defer_writes_after_reads:
            return self.io_stream
        if self._write_stream is None:
            self._write_stream = torch.cuda.Stream(device=self.device, priority=0)
        return self._write_stream

    def wait_write_stream_event(self, event: torch.cuda.Event) -> None:
        """Order later write batches after ``event`` on the device; the host does not block."""
        if self.pool is not None and self.pool.device.type == "cuda":
            self.write_stream.wait_event(event)

    def bind(self, pool: torch.Tensor) -> None:
        """Bind the engine's paged KV pool (direct mode registers it with the store once)."""
        self.pool = pool
        self.layers = None
        if not self.staged:
            self.store.register_pool(pool)

    def bind_layers(self, layers: Sequence[torch.Tensor]) -> None:
        """Bind one KV tensor per layer, ``[planes, num_blocks, block, heads, dim]`` (vLLM's layout)."""
        self.layers = list(layers)
        self.pool = self.layers[0]
        if not self.staged:
            self.store.register_layers(self.layers)

    # -- staged (host-side) gather/scatter ------------------------------------
    def _layer_views(self):
        if getattr(self, "layers", None):
            return self.layers
        return [self.pool[i] for i in range(self.pool.shape[0])]

    def _gather_chunks(self, bt: np.ndarray) -> torch.Tensor:
        """Blocks -> bytes laid out like chunk segments: [chunk][layer][block][plane]."""
        layers = self._layer_views()
        idx = torch.from_numpy(bt.reshape(-1)).to(layers[0].device)
        per_layer = [t[:, idx] for t in layers]  # [P, n*bpc, ...]
        x = torch.stack(per_layer, 0)  # [L, P, n*bpc, ...]
        n, bpc = bt.shape
        x = x.reshape(x.shape[0], x.shape[1], n, bpc, *x.shape[3:]).permute(2, 0, 3, 1, *range(4, x.dim() + 1))
        return x.contiguous().view(torch.uint8).reshape(n, -1)

    def _scatter_chunks(self, data: torch.Tensor, bt: np.ndarray) -> None:
        layers = self._layer_views()
        n, bpc = bt.shape
        P = layers[0].shape[0]
        tail = layers[0].shape[2:]
        x = data.reshape(-1).view(layers[0].dtype).reshape(n, len(layers), bpc, P, *tail)
        idx = torch.from_numpy(bt.reshape(-1)).to(layers[0].device)
        for li, t in enumerate(layers):
            t[:, idx] = x[:, li].permute(2, 0, 1, *range(3, x.dim() - 1)).reshape(P, n * bpc, *tail).to(t.device)

    # -- restores -------------------------------------------------------------
    def _table(self, block_table) -> np.ndarray:
        bt = block_table.cpu().numpy() if isinstance(block_table, torch.Tensor) else np.asarray(block_table)
        return bt.reshape(-1, self.geometry.blocks_per_chunk).astype(np.int64)

    def start_read_plan(self, keys: Sequence[bytes], block_table, layers: Sequence[int] | None = None,
                        window: int = 4) -> LayerwiseReadPlan:
        """Restore ``keys`` (chunk order) into ``block_table`` rows, layer by layer."""
        if self.pool is None:
            raise RuntimeError("bind() the KV pool first")
        layers = list(range(self.geometry.num_layers)) if layers is None else list(layers)
        if self.staged:
            from ..common.errors import DirectTransferUnavailable

            raise DirectTransferUnavailable("layerwise plans need a direct (paged) store")
        if self.pool.device.type != "cuda":
            return _WholeRestorePlan(self.load(keys, block_table, layers))  # host pool: no streams to overlap
        self.stats["read_chunks"] += len(keys)
        return LayerwiseReadPlan(self, keys, self._table(block_table), layers, self.io_stream, window)

    @property
    def host_gated_layer_waits(self) -> bool:
        """Layer waits block the host instead of the consumer stream (``TUTTI_LAYER_WAIT=host``).

        The default is a device-side wait: the consumer stream waits on the
        restore's event and the host runs ahead. The host-gated form launches
        layer l's consumer work only after the host saw layer l restored.
        """
        return (text("TUTTI_LAYER_WAIT") or "").strip().lower() == "host"

    @property
    def split_completion(self) -> bool:
        """Reads finish in a drain launched on the consumer's stream (or by the host fallback)."""
        opts = getattr(self.store, "runtime_options", None) or {}
        return bool(opts.get("async_completion")) or flag("TUTTI_ASYNC_COMPLETION")

    def load(self, keys: Sequence[bytes], block_table, layers: Sequence[int] | None = None):
        """Restore all (or ``layers``) of ``keys`` in one submission; returns a completion with ``read_ms()``."""
        bt = self._table(block_table)
        if not self.staged and self.pool.device.type != "cuda":
            # a direct store serving host memory (e.g. the POSIX backend): host-executed, host-timed
            self.stats["read_chunks"] += len(keys)
            t0 = time.perf_counter()
            comp = self.store.get_paged(keys, bt, layers=layers, stream=None)
            comp.wait()
            return TimedCompletion(comp, device_timed=False, host_ms=(time.perf_counter() - t0) * 1e3)
        if not self.staged:
            self.stats["read_chunks"] += len(keys)
            s = self.io_stream
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record(s)
            comp = self.store.get_paged(keys, bt, layers=layers, stream=s)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record(s)
            return TimedCompletion(comp, ev0, ev1, device_timed=not self.split_completion)
        t0 = time.perf_counter()
        comp = self._staged_load(keys, bt)
        return TimedCompletion(comp, device_timed=False, host_ms=(time.perf_counter() - t0) * 1e3)

    def _staging(self, direction: str) -> StagingBuffer:
        buf = self._staging_bufs.get(direction)
        if buf is None:
            buf = self._staging_bufs[direction] = StagingBuffer(self.store, self.geometry.chunk_bytes, self.pool.device)
        return buf

    def _staged_load(self, keys, bt):
        g = self.geometry
        dev = self.pool.device
        with self._staging("load").use(len(keys)) as (staging, bid, _):
            comp = self.store.get_batch([(k, bid, i * g.chunk_bytes) for i, k in enumerate(keys)])
            comp.wait()
            if dev.type == "cuda" and not getattr(self, "layers", None):
                from .. import ops

                ops.scatter_blocks(staging, self.pool, torch.from_numpy(bt.reshape(-1)), g.blocks_per_chunk)
            else:
                self._scatter_chunks(staging, bt)
        return comp

    # -- stores ---------------------------------------------------------------
    def plan_store(self, keys: Sequence[bytes]) -> StorePlan | None:
        plan = self.index.plan_store(keys)
        if plan is not None and plan.evicted_keys and hasattr(self.store, "drop"):
            self.store.drop(plan.evicted_keys)  # capacity closure: the index decided, the store executes
            self.stats["evicted_chunks"] += len(plan.evicted_keys)
        return plan

    def store_chunks(self, keys: Sequence[bytes], block_table, *, after: torch.cuda.Event | None = None):
        """Persist chunks ``keys`` from ``block_table`` rows once ``after`` (compute) has happened."""
        keys = [bytes(k) for k in keys]
        plan = self.plan_store(keys)
        if plan is None:
            self.stats["store_refused"] += 1
            return None
        new = set(plan.new_keys)
        idx = [i for i, k in enumerate(keys) if k in new]
        if not idx:
            return None
        bt = self._table(block_table)[idx]
        wkeys = [keys[i] for i in idx]
        on_gpu = self.pool is not None and self.pool.device.type == "cuda"
        stream = self.write_stream if on_gpu else None
        if stream is not None:
            if after is not None:
                stream.wait_event(after)
            else:
                stream.wait_stream(torch.cuda.current_stream(self.device))

        def settle(inner):
            return PostCompletion(inner, after=lambda: self.index.confirm_store(wkeys, True),
                                  on_error=lambda: self.index.confirm_store(wkeys, False))

        if not self.staged:
            comp = settle(self.store.put_paged(wkeys, bt, stream=stream))
        else:
            g = self.geometry
            with self._staging("store").use(len(wkeys)) as (staging, bid, holder):
                if on_gpu and not getattr(self, "layers", None):
                    from .. import ops

                    with torch.cuda.stream(stream):
                        ops.gather_blocks(self.pool, torch.from_numpy(bt.reshape(-1)), g.blocks_per_chunk,
                                          out=staging)
                    stream.synchronize()
                else:
                    if on_gpu:
                        stream.synchronize()
                    staging.copy_(self._gather_chunks(bt).reshape(-1))
                comp = settle(self.store.put_batch([(k, bid, i * g.chunk_bytes) for i, k in enumerate(wkeys)]))
                holder["pending"] = comp  # the store may read the buffer until this batch completes
        self._writes.append(comp)
        self.stats["write_chunks"] += len(wkeys)
        return comp

    def poll_writes(self) -> int:
        done = 0
        while self._writes and self._writes[0].query():
            try:
                self._writes.popleft().wait()
            except Exception as e:  # noqa: BLE001
                LOG.warning("write failed: %s", e)
            done += 1
        self._maybe_checkpoint()
        return done

    def wait_idle(self, timeout_s: float | None = None) -> None:
        """Settle the queued writes; with ``timeout_s``, writes still running then are dropped (not committed)."""
        from .completion import settle_by

        deadline = None if timeout_s is None else time.monotonic() + float(timeout_s)
        while self._writes:
            try:
                if not settle_by(self._writes[0], deadline):
                    LOG.warning("%d write(s) still running after %.0f s; left uncommitted", len(self._writes), timeout_s)
                    self._writes.clear()
                    break
            except Exception as e:  # noqa: BLE001
                LOG.warning("write failed: %s", e)
            if self._writes:
                self._writes.popleft()
        self._maybe_checkpoint(force=False)

    def _maybe_checkpoint(self, force: bool = False) -> None:
        if not hasattr(self.store, "objects") or self.store.objects is None:
            return
        now = time.monotonic()
        periodic = self._checkpoint_interval > 0  # 0 turns periodic checkpoints off (TUTTI_CHECKPOINT_INTERVAL_S=0)
        if force or (periodic and now - self._last_checkpoint >= self._checkpoint_interval):
            self.store.objects.checkpoint()
            self._last_checkpoint = now
