"""Worker side of the vLLM connector: per-step loads and saves on one TP rank.

* ``register_kv_caches``: binds vLLM's per-layer KV tensors
  (``[2, num_blocks, block_size, kv_heads, head_dim]``) to the engine once.
* ``start_load_kv``: one layerwise read plan for all synchronous loads of the
  step (layer l's restore overlaps layer l-1's attention); asynchronous loads
  are submitted as whole-prefix restores and reported by ``get_finished``.
* ``wait_for_layer_load``: device-side wait of the current stream on layer l.
* ``wait_for_save``: settles the loads (TP failure consensus: every rank
  agrees on the failed chunk range), then queues this step's new full chunks
  for persisting behind the forward's compute event and returns: the step
  does not wait for its saves. Saves that finished since (checked without
  blocking here and in ``get_finished``) are committed then (payload, then
  header) and reported committed in that step's metadata. At most
  ``max_inflight_saves`` saves stay in flight; beyond that the oldest is
  waited for (back-pressure).
* Block reuse after a request finishes: vLLM frees its blocks at once. A
  save of them may still be queued on the device, so the next step names the
  request (``finished_saving``) and ``start_load_kv`` makes the compute stream
  wait for the save kernels' device events before the forward that may write
  those blocks again: ordering on the device, no host wait.
* ``get_finished``: finished asynchronous loads (``finished_recving``).
* Measurements for the scheduler's load policy, harvested without blocking
  (a sample whose events have not completed waits for a later step):
  ``read_samples`` (chunks, device ms) of finished restores and
  ``step_samples`` (tokens, device ms) of forwards without a synchronous read.
Parity: reference tutti/integration/vllm/worker.py:461-1822 (WorkerImpl,
start_load_kv, wait_for_layer_load, save_kv_layer, wait_for_save,
_synchronize_load_failure, async loads).
"""
from __future__ import annotations

import logging
import re
import time
from collections import deque
from typing import Callable

import numpy as np
import torch

from ...common.observability import HealthReporter
from ...engine.completion import LoadGateError
from ...engine.core import KVEngine
from ...engine.entities import EntityEngines
from ...parallel.tp_consensus import ChunkFailure, TpFailureConsensus
from .metadata import LoadSpec, TuttiConnectorMetadata, TuttiWorkerMetadata

LOG = logging.getLogger("tutti_b200.vllm")
_LAYER_RE = re.compile(r"(\d+)")


class _FailedLoad:
    """A load that failed at submission; raises when settled."""

    def __init__(self, error: BaseException):
        self.error = error

    def wait(self) -> None:
        raise self.error


def _dense(x: torch.Tensor) -> bool:
    """True when ``x`` covers a gap-free range of its storage (any dimension order)."""
    expected = 1
    for stride, size in sorted(zip(x.stride(), x.shape)):
        if size == 1:
            continue
        if stride != expected:
            return False
        expected *= size
    return True


def _contiguous_view(t: torch.Tensor, shape: tuple[int, ...]) -> torch.Tensor:
    strides, acc = [], 1
    for n in reversed(shape):
        strides.append(acc)
        acc *= n
    return torch.as_strided(t, shape, tuple(reversed(strides)), t.storage_offset())


def normalize_kv_layer(t: torch.Tensor) -> torch.Tensor:
    """A contiguous ``[planes, num_blocks, block, heads, dim]`` view of one layer's KV cache bytes.

    vLLM attention backends lay the cache out as ``[2, num_blocks, block, heads,
    dim]`` (K and V planes first), ``[num_blocks, 2, block, heads, dim]`` (K and V
    of a block together) or ``[num_blocks, block, dim]`` (MLA latents), and may
    permute the dimensions inside a block (e.g. heads before tokens). Only bytes
    move: each block (or plane-block) must be one gap-free range at a fixed
    stride, and the view below addresses exactly those bytes; a block-major
    layout becomes one plane whose block holds K and V together.
    """
    if t.dim() == 5 and t.shape[0] == 2 and t.shape[1] != 2:
        nb = t.shape[1]
        per = t[0, 0].numel()
        if _dense(t[0, 0]) and t.stride(1) == per and t.stride(0) == nb * per:
            return _contiguous_view(t, tuple(t.shape))
    elif t.dim() == 5 and t.shape[1] == 2:
        nb, _, bs, heads, dim = t.shape
        if _dense(t[0]) and t.stride(0) == t[0].numel():
            return _contiguous_view(t, (1, nb, bs, 2 * heads, dim))
    elif t.dim() == 3:
        nb, bs, dim = t.shape
        if _dense(t[0]) and t.stride(0) == t[0].numel():
            return _contiguous_view(t, (1, nb, bs, 1, dim))
    raise ValueError(f"unsupported KV cache layout {tuple(t.shape)} with strides {t.stride()}")


def entity_tag(name: str) -> str:
    """The part of a layer name after its layer number (``self_attn.indexer.k_cache``)."""
    m = re.search(r"\d+\.(.*)$", name)
    tag = (m.group(1) if m else name) or "entity"
    return re.sub(r"[^A-Za-z0-9_.-]", "_", tag)


def layer_index(name: str) -> int:
    m = _LAYER_RE.findall(name)
    if not m:
        raise ValueError(f"cannot find a layer index in {name!r}")
    return int(m[0])


def fanout_items(keys, blocks, blocks_per_chunk: int, groups):
    """Restore items of one step's loads for every TP rank (``groups[r]``: rank r's replica group).

    Rank r's copy of chunk i lands in the same block ids on every rank (vLLM's
    block table is shared by the TP group). A rank alone in its group reads its
    own slice (source = itself); in a larger group every member's item names the
    chunk's owner (``replica_owner``), so the group's copies share one read.
    """
    from ...parallel.fanout import RestoreItem
    from ...parallel.replica_layout import replica_owner

    bpc = int(blocks_per_chunk)
    out = []
    for r, g in enumerate(groups):
        for i, k in enumerate(keys):
            src = None if len(g) == 1 else replica_owner(k, g)
            out.append(RestoreItem(rank=r, key=bytes(k), block_ids=[int(b) for b in blocks[i * bpc:(i + 1) * bpc]],
                                   source=src))
    return out


class WorkerSide:
    def __init__(self, make_engine: Callable[..., KVEngine], *, block_size: int,
                 chunk_tokens: int, tp_rank: int = 0, tp_size: int = 1,
                 consensus: TpFailureConsensus | None = None, failure_policy: str = "recompute",
                 lookahead: int = 4, max_inflight_saves: int = 64, replica_io: bool = False, group=None,
                 replica_kind: str = "main", kv_heads: int | None = None, replica_io_saves: str = "local"):
        if failure_policy not in ("recompute", "fail"):
            raise ValueError("kv_load_failure_policy must be recompute or fail")
        self.make_engine = make_engine
        self.block_size = block_size
        self.chunk_tokens = chunk_tokens
        self.blocks_per_chunk = chunk_tokens // block_size
        self.tp_rank = tp_rank
        self.tp_size = tp_size
        self.consensus = consensus or TpFailureConsensus()
        self.failure_policy = failure_policy
        self.lookahead = max(1, int(lookahead))  # layers read ahead of the layer attention waits for
        self.engine: KVEngine | None = None
        self.health: HealthReporter | None = None
        self.layer_of: dict[str, int] = {}
        self._plan = None
        self._plan_loads: list[LoadSpec] = []
        self._async: dict[str, tuple[object, LoadSpec, float]] = {}
        self._finished_recv: set[str] = set()
        self._load_error_blocks: set[int] = set()
        self._meta = TuttiWorkerMetadata()
        self._read_timing: list[tuple[int, object]] = []  # (chunks, plan or completion with read_ms())
        self._step_timing: list[tuple[object, object, int]] = []  # (start, end, tokens) of steps w/o sync reads
        self._step: tuple[object, int, bool] | None = None  # this step's start event, tokens, had sync loads
        self.max_inflight_saves = max(1, int(max_inflight_saves))
        # replica_io: each GPU reads the chunks on the drives affine to it for every TP rank
        # and its io kernel stores each rank's slice into that rank's caches over NVLink
        self.replica_io = bool(replica_io) and tp_size > 1
        self.group = group
        # which ranks hold identical copies (duplicated KV heads, an MLA latent cache):
        # a chunk of such a cache is read once, by its owner's affine GPU, for the group
        self.replica_kind = replica_kind
        self.kv_heads = kv_heads
        self._replica_groups = [(r,) for r in range(tp_size)]
        # replica_io_saves="fanin": a step's saves are written by the drive-affine GPUs, which
        # gather every rank's blocks over NVLink; commits are decided together (store_harvest)
        if replica_io_saves not in ("local", "fanin"):
            raise ValueError("replica_io_saves must be local or fanin")
        self.replica_io_saves = replica_io_saves
        self._fanin_on = False
        self._save_board = None
        self._fanin: dict = {}  # batch id -> FaninBatch not yet decided (the same ids on every rank)
        self._fanin_of: dict[str, set[int]] = {}  # request id -> undecided batches holding its saves
        self._fanin_next = 0
        self._fan = None
        self._board = None
        self._epoch = 0
        self._saves: deque = deque()  # (SaveSpec, completion) in submission order
        self._saves_of: dict[str, int] = {}  # request id -> saves in flight on this rank
        self._save_events: dict[str, list] = {}  # request id -> device events after its save kernels

    # -- binding --------------------------------------------------------------
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]) -> None:
        names = sorted(kv_caches, key=lambda n: (layer_index(n), n))
        self.layer_of = {n: i for i, n in enumerate(names)}
        views = {n: normalize_kv_layer(kv_caches[n]) for n in names}
        # entities: layers whose pages share one shape and dtype (main KV, index cache, ...)
        groups: dict[tuple, list[str]] = {}
        for n in names:
            t = views[n]
            groups.setdefault((t.shape[0],) + tuple(t.shape[2:]) + (t.dtype,), []).append(n)
        if len(groups) == 1:
            self.engine = self.make_engine([views[n] for n in names])
            if self.replica_io:
                self._setup_fanout([views[n] for n in names])
            return
        ordered = sorted(groups.values(), key=len, reverse=True)  # the main KV has the most layers
        engines, where = [], {}
        for e, members in enumerate(ordered):
            tag = "" if e == 0 else entity_tag(members[0])
            engines.append(self.make_engine([views[n] for n in members], tag))
            for li, n in enumerate(members):
                where[n] = (e, li)
        self.engine = EntityEngines(engines, [where[n] for n in names], [entity_tag(g[0]) for g in ordered])

    def _setup_fanout(self, layers) -> None:
        """Peer mappings of every rank's per-layer caches and a ready-flag board (collective)."""
        from ...parallel.fanout import FanoutRestorer, PeerLayers, ReadyBoard

        store = self.engine.store
        if not hasattr(store, "restore_placements") or self.engine.staged:
            LOG.warning("[tutti] replica_io needs the direct (paged) NVMe store; each rank restores its own slice")
            self.replica_io = False
            return
        from ...parallel.replica_layout import replica_group, validate_replica_io

        if self.kv_heads:
            try:
                validate_replica_io(self.tp_size, int(self.kv_heads))
                self._replica_groups = [replica_group(r, self.tp_size, int(self.kv_heads), self.replica_kind)
                                        for r in range(self.tp_size)]
            except ValueError as e:
                LOG.warning("[tutti] replica_io: %s; every rank's slice is read on its own", e)
        self._peers = PeerLayers(layers, self.group)
        self._fan = FanoutRestorer(store, self._peers, self.group)
        self._board = ReadyBoard(layers[0].device.index, self.group, slots=len(layers))
        self._n_drives = max(1, len(getattr(store, "mounts", [None])))
        self._affine = list(range(self.tp_size))
        if self.replica_io_saves == "fanin":
            # slot 0: every rank's forward of batch E wrote its blocks; slot 1: every GPU's writes of E ended
            self._save_board = ReadyBoard(layers[0].device.index, self.group, slots=2)
            self._fanin_on = True

    # -- loads ----------------------------------------------------------------
    def start_load_kv(self, meta: TuttiConnectorMetadata) -> None:
        self._meta = TuttiWorkerMetadata()
        # blocks of requests that finished may be written by this step's forward:
        # it follows their save kernels on the device
        for rid in getattr(meta, "finished_saving", ()) or ():
            for ev in self._save_events.pop(rid, ()):
                torch.cuda.current_stream().wait_event(ev)
            # fan-in saves: until every GPU's writes of the request's batches ended (device wait,
            # bounded; a wait that gives up fails the batch, so nothing torn is committed)
            for bid in sorted(self._fanin_of.pop(rid, ())):
                b = self._fanin.get(bid)
                if b is not None:
                    cs = torch.cuda.current_stream() if torch.cuda.is_available() else None
                    b.reuse_tickets.append(self._save_board.wait(1, bid, cs))
        if self.engine is not None:
            if self.health is None:
                self.health = HealthReporter(self.engine.store)
            self.health.maybe_log()
        sync = [l for l in meta.loads if not l.is_async]
        if torch.cuda.is_available():
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._step = (ev, int(getattr(meta, "step_tokens", 0)), bool(sync))
        for spec in meta.loads:
            if spec.is_async:
                comp = self.engine.load(spec.keys, np.asarray(spec.block_ids, dtype=np.int64))
                self._async[spec.request_id] = (comp, spec, time.perf_counter())
        self._plan_loads = sync
        self._plan = None
        if sync:
            keys = [k for s in sync for k in s.keys]
            blocks = np.asarray([b for s in sync for b in s.block_ids], dtype=np.int64)
            try:
                if self._fan is not None:
                    self._plan = self._start_fanout_plan(keys, blocks)
                elif self.engine.staged:
                    self._plan = self.engine.load(keys, blocks)
                else:
                    self._plan = self.engine.start_read_plan(keys, blocks, window=self.lookahead)
            except Exception as e:  # noqa: BLE001 - settled (with TP consensus) in wait_for_save
                self._plan = _FailedLoad(e)

    def _start_fanout_plan(self, keys, blocks):
        from ...parallel.fanout import FanoutLayerPlan

        items = fanout_items(keys, blocks, self.blocks_per_chunk, self._replica_groups)
        self._epoch += 1
        return FanoutLayerPlan(self._fan, self._board, items, self._n_drives, self._affine,
                               list(range(self.engine.geometry.num_layers)), self.engine.io_stream, self._epoch,
                               window=self.lookahead)

    def wait_for_layer_load(self, layer_name: str) -> None:
        if self._plan is not None and hasattr(self._plan, "wait_layer"):
            self._plan.wait_layer(self.layer_of[layer_name])

    def _settle_sync_loads(self, generation: int) -> None:
        if self._plan is None:
            return
        local: list[ChunkFailure] = []
        try:
            if hasattr(self._plan, "finish"):
                self._plan.finish()
            else:
                self._plan.wait()
        except (LoadGateError, Exception) as e:  # noqa: BLE001 - mapped to chunk failures below
            failed = getattr(e, "failed_chunks", None) or range(sum(len(s.keys) for s in self._plan_loads))
            base = 0
            for ordinal, spec in enumerate(self._plan_loads):
                mine = [c - base for c in failed if base <= c < base + len(spec.keys)]
                if mine:
                    local.append(ChunkFailure(ordinal, min(mine), max(mine) - min(mine) + 1))
                base += len(spec.keys)
        if not local and hasattr(self._plan, "read_ms"):
            self._read_timing.append((sum(len(s.keys) for s in self._plan_loads), self._plan))
        cons = self.consensus.coordinate(generation, len(self._plan_loads), local)
        if cons.failed:
            if self.failure_policy == "fail":
                raise LoadGateError(f"KV load failed on some TP rank: {cons.failures}")
            self.consensus.drain_barrier(generation, True)
            for f in cons.failures:
                spec = self._plan_loads[f.request]
                first_tok = f.first_chunk * self.chunk_tokens
                self._meta.failed_loads[spec.request_id] = first_tok
                # every block from the first failed chunk on must be recomputed
                self._load_error_blocks.update(spec.block_ids[f.first_chunk * self.blocks_per_chunk:])
        self._plan = None

    # -- saves ----------------------------------------------------------------
    def _harvest_samples(self) -> None:
        """Move finished read and step timings into this step's metadata (never blocks)."""
        keep = []
        for chunks, src in self._read_timing[-64:]:
            ms = src.read_ms()
            if ms is None:
                keep.append((chunks, src))
            elif chunks > 0 and ms > 0:
                self._meta.read_samples.append((chunks, ms))
        self._read_timing = keep
        pending = []
        for start, end, tokens in self._step_timing[-64:]:
            if not end.query():
                pending.append((start, end, tokens))
            elif tokens > 0:
                self._meta.step_samples.append((tokens, float(start.elapsed_time(end))))
        self._step_timing = pending

    def wait_for_save(self, meta: TuttiConnectorMetadata) -> TuttiWorkerMetadata:
        self._meta.generation = meta.generation
        if self._step is not None:
            start, tokens, had_sync = self._step
            self._step = None
            if not had_sync:  # a synchronous read's stall says nothing about compute
                end = torch.cuda.Event(enable_timing=True)
                end.record()
                self._step_timing.append((start, end, tokens))
        self._settle_sync_loads(meta.generation)
        if self._fanin_on:
            if meta.saves:
                self._fanin_begin(meta.saves)
            if self._fanin:
                # back-pressure: past max_inflight_saves undecided batches every rank waits for its
                # own writes (the condition is the same on every rank: they hold the same batches)
                self._fanin_harvest(blocking=len(self._fanin) > self.max_inflight_saves)
            self._harvest_samples()
            return self._meta
        if meta.saves:
            ev = torch.cuda.Event() if torch.cuda.is_available() and not self.engine.staged else None
            if ev is not None:
                ev.record()
            for spec in meta.saves:
                comp = self.engine.store_chunks(spec.keys, np.asarray(spec.block_ids, dtype=np.int64), after=ev)
                if comp is None:  # nothing new to write: resident chunks count as committed
                    self._count_resident(spec.keys)
                    continue
                ws = getattr(self.engine, "write_stream", None) if ev is not None else None
                if ws is not None:
                    done = torch.cuda.Event()
                    done.record(ws)  # behind the save kernel on the engine's write stream
                    self._save_events.setdefault(spec.request_id, []).append(done)
                self._saves.append((spec, comp))
                self._saves_of[spec.request_id] = self._saves_of.get(spec.request_id, 0) + 1
            while len(self._saves) > self.max_inflight_saves:
                self._settle_save(*self._saves.popleft())
        self._harvest_saves()
        self._harvest_samples()
        return self._meta

    # -- fan-in saves (replica_io_saves="fanin") ---------------------------------------------
    def _fanin_begin(self, saves) -> None:
        """Start one batch for this step's saves (collective: every rank, same step, same specs)."""
        self._fanin_next += 1
        bid = self._fanin_next
        stream = torch.cuda.current_stream() if torch.cuda.is_available() else None
        self._save_board.signal(0, bid, stream)  # this rank's forward wrote the blocks
        keys, blocks = [], []
        for spec in saves:
            keys += [bytes(k) for k in spec.keys]
            blocks += list(spec.block_ids)
        plan = self.engine.plan_store(keys)  # this rank's index: capacity closure, pending keys
        mine = list(plan.new_keys) if plan is not None else []
        items = fanout_items(keys, np.asarray(blocks, dtype=np.int64), self.blocks_per_chunk,
                             [(r,) for r in range(self.tp_size)])
        b = self._fan.store_begin(bid, items, mine, self._n_drives, self._affine, self._save_board,
                                  getattr(self.engine, "write_stream", None))
        b.all_keys, b.index_keys = keys, mine
        self._fanin[bid] = b
        for spec in saves:
            self._fanin_of.setdefault(spec.request_id, set()).add(bid)

    def _fanin_harvest(self, blocking: bool = False) -> None:
        """Commit or abort the batches every rank finished (collective, lockstep on all ranks)."""
        for b in self._fan.store_harvest(list(self._fanin.values()), self._save_board, blocking):
            del self._fanin[b.batch_id]
            self.engine.index.confirm_store(getattr(b, "index_keys", b.keys), bool(b.committed))
            if b.committed:
                for k in b.keys:
                    self._meta.committed[k] = self._meta.committed.get(k, 0) + 1
            else:
                LOG.warning("fan-in save batch %d aborted: %s", b.batch_id, b.error or "a peer failed")
            self._count_resident(getattr(b, "all_keys", ()))

    def _count_resident(self, keys) -> None:
        for k in keys:
            if k not in self._meta.committed and self.engine.index.is_resident(k):
                self._meta.committed[k] = 1

    def _settle_save(self, spec, comp) -> None:
        """Wait for (or collect) one save, commit it and count its chunks in this step's metadata."""
        try:
            comp.wait()
        except Exception as e:  # noqa: BLE001 - a failed save only costs a future recompute
            LOG.warning("save of %d chunk(s) for %s failed: %s", len(spec.keys), spec.request_id, e)
        else:
            for k in spec.keys:
                self._meta.committed[k] = self._meta.committed.get(k, 0) + 1
        self._count_resident(spec.keys)  # chunks another save made resident meanwhile
        left = self._saves_of.get(spec.request_id, 1) - 1
        if left > 0:
            self._saves_of[spec.request_id] = left
        else:
            self._saves_of.pop(spec.request_id, None)

    def _harvest_saves(self) -> None:
        """Commit the saves whose device work has finished; never blocks on one in flight."""
        if not self._saves:
            return
        pending = deque()
        for spec, comp in self._saves:
            if comp.query():
                self._settle_save(spec, comp)
            else:
                pending.append((spec, comp))
        self._saves = pending

    def saves_in_flight(self) -> int:
        return len(self._saves)

    def settle_saves(self, timeout_s: float | None = None) -> int:
        """Wait for the saves in flight and commit them (reported in the next step's metadata).

        Not needed by vLLM's step loop (commits are harvested without blocking);
        for shutdown and for callers that must see their chunks committed now.
        With ``timeout_s``, saves still running at the deadline are left
        uncommitted (their chunks are simply not persisted) instead of waited
        for. Returns how many saves were settled.
        """
        n = 0
        deadline = None if timeout_s is None else time.monotonic() + float(timeout_s)
        while self._saves:
            spec, comp = self._saves[0]
            if deadline is not None:
                while not comp.query() and time.monotonic() < deadline:
                    time.sleep(0.001)
                if not comp.query():
                    LOG.warning("[tutti] %d save(s) still running after %.0f s; left uncommitted",
                                len(self._saves), timeout_s)
                    break
            self._saves.popleft()
            self._settle_save(spec, comp)
            n += 1
        return n

    # -- completion reporting -------------------------------------------------
    def get_finished(self, finished_req_ids: set[str]) -> tuple[set[str] | None, set[str] | None]:
        self._harvest_saves()
        done = set()
        for rid, (comp, spec, t0) in list(self._async.items()):
            if comp.query():
                try:
                    comp.wait()
                    if hasattr(comp, "read_ms"):
                        self._read_timing.append((len(spec.keys), comp))
                except Exception:  # noqa: BLE001
                    self._load_error_blocks.update(spec.block_ids)
                    self._meta.failed_loads[rid] = 0
                done.add(rid)
                del self._async[rid]
        return None, (done or None)

    def get_block_ids_with_load_errors(self) -> set[int]:
        out, self._load_error_blocks = self._load_error_blocks, set()
        return out

    def shutdown(self, timeout_s: float = 120.0) -> None:
        """Settle saves and loads, then close the store; nothing waits past ``timeout_s`` in all."""
        from ...engine.completion import settle_by

        deadline = time.monotonic() + float(timeout_s)
        left = lambda: max(0.0, deadline - time.monotonic())  # noqa: E731
        self.settle_saves(left())
        # undecided fan-in batches: no collective at shutdown (peers may be gone); their
        # writes are waited for (no DMA outlives the caches) and this rank's keys aborted
        for b in list(self._fanin.values()):
            try:
                if b.comp is not None:
                    settle_by(b.comp, deadline)
            except Exception:  # noqa: BLE001
                pass
            if b.keys:
                self.engine.store.objects.abort(b.keys)
            self.engine.index.confirm_store(getattr(b, "index_keys", b.keys), False)
        self._fanin.clear()
        if self._save_board is not None:
            self._save_board.close()
        if self._board is not None:
            self._board.close()
            self._peers.close()
        for comp, _, _ in self._async.values():
            try:
                settle_by(comp, deadline)
            except Exception:  # noqa: BLE001
                pass
        self._async.clear()
        if self.engine is not None:
            self.engine.wait_idle(left())
            if hasattr(self.engine.store, "close"):
                try:
                    self.engine.store.close(left())
                except TypeError:  # a store whose close takes no deadline
                    self.engine.store.close()
