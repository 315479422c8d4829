"""TuttiKVStore: the native-runtime-backed KV store.

It owns
  * an ``ObjectLayout`` (segment-file object store: which slot holds a chunk),
  * a native runtime (``nvme-gpu``: GPU-initiated NVMe through emulated or
    real controllers with the paged scatter fused into the io kernel; or
    ``posix``: host-executed pread/pwrite, the CPU-centric baseline),
  * a target-ticket cache (segment file -> runtime target handle),
  * registered memory (the engine's whole paged KV pool, registered once).

Paged IO (``get_paged`` / ``put_paged``) turns (chunk keys, block table,
layers) into byte-range requests with vectorised numpy arithmetic and hands
them to ``Runtime.submit_arrays`` in one call; the runtime coalesces adjacent
target ranges into NVMe commands and the io kernel scatters each command's
pieces into the pool. Rejected requests (queue leases busy) are resubmitted
after the oldest in-flight batch drains.
Parity: reference tutti/storage/tutti_nvme/store.py:203-1125 (direct paged
backends), :1590-2830 (TuttiKVStore, _submit_retry, completions) and
layerwise_direct.py:45-181 (block table -> page requests).
"""
from __future__ import annotations

import collections
import threading
import time
from pathlib import Path
from typing import Sequence

import numpy as np
import torch

from .._native import core
from ..common.env import integer, prp_mode, runtime_option_defaults
from ..common.observability import metrics, nvtx_range
from ..models.kv_geometry import KVGeometry
from .base import StoreIOError
from .object_layout import DEFAULT_SEGMENT_FILE_SLOTS, DEFAULT_SEGMENT_HEADER_BYTES, ObjectLayout


STORED_FORMATS = ("native", "fp8_block128")


def stored_geometry(g: KVGeometry, stored_format: str = "native") -> dict:
    """On-disk sizes of one rank's chunk slice in ``stored_format``.

    ``native`` stores the pool's bytes as they are (a layer segment padded to
    4 KiB). ``fp8_block128`` stores each
    bf16 (layer, plane, block) page as E4M3 values followed by one fp32 scale per
    128 values (33/64 of the bytes; the io kernel quantises on store and
    dequantises on restore); each layer segment is padded to 4 KiB.
    """
    if stored_format == "native":
        # sub-sector pages (e.g. 8,448-byte index-cache pages) are fine; the segment is padded to 4 KiB
        if g.segment_bytes % 512:
            raise ValueError("a layer segment must be a whole number of 512-byte sectors")
        return {"plane_bytes": g.plane_block_bytes, "block_layer_bytes": g.block_layer_bytes,
                "segment_bytes": (g.segment_bytes + 4095) // 4096 * 4096, "transform": 0}
    if stored_format != "fp8_block128":
        raise ValueError(f"stored_format must be one of {STORED_FORMATS}")
    if g.dtype != torch.bfloat16 or g.plane_block_bytes % 1024:
        raise ValueError("fp8_block128 needs bf16 pages of a multiple of 512 values")
    plane = g.plane_block_bytes // 64 * 33
    block_layer = g.planes * plane
    payload = g.blocks_per_chunk * block_layer
    if payload % 512:
        raise ValueError("fp8_block128: a layer segment must be a whole number of 512-byte sectors")
    return {"plane_bytes": plane, "block_layer_bytes": block_layer,
            "segment_bytes": (payload + 4095) // 4096 * 4096, "transform": 1}


class NativeCompletion:
    """Completion of one or more runtime IOs; ``wait`` raises StoreIOError on failure."""

    def __init__(self, runtime, ios: list[int], on_success=None, on_failure=None, nbytes: int = 0,
                 kind: str = "restore"):
        self._rt = runtime
        self.kind = kind
        self._ios = list(ios)
        self._on_success = on_success
        self._on_failure = on_failure
        self._done = False
        self._results: list[dict] = []
        self.nbytes = nbytes
        self._t0 = time.perf_counter()
        self._latency_ms: float | None = None
        # enqueue_wait may race a host wait on another thread (e.g. a feeder's
        # window bound): handles are released, and _done set, only under this lock
        self._mu = threading.Lock()
        self._wait_mu = threading.Lock()
        self._error: StoreIOError | None = None

    def query(self) -> bool:
        if self._done:
            return True
        done = all(self._rt.query_io(io) != "in_flight" for io in self._ios)
        if done and self._latency_ms is None:
            self._latency_ms = (time.perf_counter() - self._t0) * 1e3
        return done

    def enqueue_wait(self, stream: torch.cuda.Stream | None = None) -> None:
        """Order ``stream`` after this batch's io kernels (no host wait)."""
        s = stream or torch.cuda.current_stream()
        with self._mu:
            if self._done:
                return  # host-waited: the data is in place
            self._rt.enqueue_wait(self._ios, s.cuda_stream)

    def wait(self, timeout_ms: int = 600_000) -> None:
        # Waiters on several threads (a feeder's window bound, a layer wait) are
        # serialised: the first settles the IOs, the others see its outcome.
        with self._wait_mu:
            if self._done:
                if self._error is not None:
                    raise self._error
                return
            try:
                self._wait_locked(timeout_ms)
            except StoreIOError as e:
                if self._done:
                    self._error = e
                raise

    def _wait_locked(self, timeout_ms: int) -> None:
        failed: list[int] = []
        kinds = set()
        results = []
        for io in self._ios:
            r = self._rt.wait(io, timeout_ms)
            if r is None:
                raise StoreIOError(f"io {io} still in flight after {timeout_ms} ms", kind="timeout")
            results.append(r)
        with self._mu:
            if self._done:
                return
            for io in self._ios:
                self._rt.release_io(io)
            self._done = True
        for r in results:
            self._results.append(r)
            if not r["ok"]:
                failed.extend(r["failed_request_indices"])
                kinds.add(r["failure_kind"])
        m = metrics()
        m.add(f"{self.kind}_ops")
        if self._latency_ms is None:
            self._latency_ms = (time.perf_counter() - self._t0) * 1e3
        m.observe(f"{self.kind}_ms", self._latency_ms)
        if failed:
            m.add("failed_ops")
            m.add("failed_requests", len(failed))
        else:
            m.add(f"{self.kind}_bytes", self.nbytes)
        if failed:
            if self._on_failure:
                self._on_failure()
            raise StoreIOError(f"{len(failed)} request(s) failed ({', '.join(sorted(kinds))})", failed,
                               ",".join(sorted(kinds)))
        if self._on_success:
            self._on_success()

    @property
    def results(self) -> list[dict]:
        return self._results


class TuttiKVStore:
    def __init__(self, root: str | Path, geometry: KVGeometry, *, capacity_chunks: int,
                 mounts: Sequence[str] | None = None, device: int = 0, rank: int = 0, rank_count: int = 1,
                 backend: str = "nvme-gpu", runtime_options: dict | None = None,
                 segment_file_slots: int = DEFAULT_SEGMENT_FILE_SLOTS,
                 segment_header_bytes: int = DEFAULT_SEGMENT_HEADER_BYTES, namespace: bytes = b"",
                 materialize: str = "zeros", max_retries: int = 1000, stored_format: str = "native"):
        self.root = Path(root)
        self.geometry = geometry
        self.device = device
        self.backend = backend
        self.mounts = [str(m) for m in (mounts or [self.root / "dev0"])]
        # emulated drives with in-memory media get a write cache: this store flushes before it commits
        self.runtime_options = {"emulator_write_back": True, **runtime_option_defaults(), **dict(runtime_options or {})}
        self.prp_mode = prp_mode()
        self.stored = stored_geometry(geometry, stored_format)
        if stored_format != "native" and backend != "nvme-gpu":
            raise ValueError(f"stored_format {stored_format!r} needs the nvme-gpu backend (fused in its io kernel)")
        fp = geometry.fingerprint() + ("" if stored_format == "native" else ":" + stored_format)
        self.layout = ObjectLayout(self.root, segment_bytes=self.stored["segment_bytes"],
                                   segment_count=geometry.num_layers, capacity_chunks=capacity_chunks,
                                   mounts=self.mounts, namespace=namespace or fp.encode(),
                                   rank=rank, rank_count=rank_count, segment_file_slots=segment_file_slots,
                                   segment_header_bytes=segment_header_bytes, materialize=materialize,
                                   precreate_min_free_bytes=integer("TUTTI_PRECREATE_MIN_FREE_BYTES"))
        self.max_retries = max_retries
        self.runtime = None
        self._targets: dict[str, int] = {}
        self._pool = None  # (tensor, handle, num_blocks)
        self._inflight: collections.deque[NativeCompletion] = collections.deque()
        self.last_submit_profile: dict = {}
        self._layer_mems = np.zeros(0, dtype=np.uint64)  # per-layer registrations, if any

    # -- lifecycle ------------------------------------------------------------
    @property
    def capacity_chunks(self) -> int:
        return self.layout.capacity_chunks

    @property
    def objects(self):
        return self.layout.store

    def open(self) -> "TuttiKVStore":
        if self.runtime is not None:
            return self
        for m in self.mounts:
            Path(m).mkdir(parents=True, exist_ok=True)
        self.layout.open()
        c = core()
        if self.backend == "nvme-gpu":
            self.runtime = c.make_emulated_nvme_runtime(self.device, self.mounts, self.runtime_options)
        elif self.backend == "posix":
            self.runtime = c.make_posix_runtime(self.device, self.mounts, self.runtime_options)
        else:
            raise ValueError(f"unknown backend {self.backend!r}")
        return self

    def close(self, timeout_s: float | None = None) -> None:
        """Settle what is in flight and shut the runtime down; with ``timeout_s`` nothing waits past it."""
        from ..engine.completion import settle_by

        deadline = None if timeout_s is None else time.monotonic() + float(timeout_s)
        for comp in list(self._inflight):
            try:
                if not settle_by(comp, deadline):
                    break  # the runtime's shutdown below reports what is still running
            except StoreIOError:
                pass
        self._inflight.clear()
        if self.runtime is not None:
            left_ms = 30_000 if deadline is None else int(max(0.0, min(30.0, deadline - time.monotonic())) * 1e3)
            try:
                self.runtime.shutdown(left_ms)
            except Exception as e:  # noqa: BLE001 - IO still running at the deadline
                import logging

                logging.getLogger("tutti_b200.store").warning("runtime shutdown: %s", e)
            self.runtime = None
        self._targets.clear()
        self._pool = None
        self.layout.close()

    def __enter__(self):
        return self.open()

    def __exit__(self, *exc):
        self.close()

    # -- memory and tickets ---------------------------------------------------
    def register_pool(self, pool: torch.Tensor) -> int:
        """Register the whole paged pool ``pool`` (shape ``geometry.pool_shape(nb)``) once."""
        g = self.geometry
        if pool.dim() != 6 or pool.shape[0] != g.num_layers or pool.shape[1] != g.planes:
            raise ValueError(f"pool shape {tuple(pool.shape)} does not match {g.name}")
        if not pool.is_contiguous():
            raise ValueError("pool must be contiguous")
        kind = "device" if pool.is_cuda else ("pinned" if pool.is_pinned() else "host")
        nbytes = pool.numel() * pool.element_size()
        h = self.runtime.register_memory(pool.data_ptr(), nbytes, kind,
                                         pool.device.index if pool.is_cuda else -1)
        self._pool = (pool, h, pool.shape[2])
        return h

    def register_layers(self, layers: Sequence[torch.Tensor]) -> list[int]:
        """Register per-layer KV tensors ``[planes, num_blocks, block, heads, dim]`` (one allocation each)."""
        g = self.geometry
        if len(layers) != g.num_layers:
            raise ValueError(f"expected {g.num_layers} layer tensors, got {len(layers)}")
        handles = []
        for t in layers:
            if t.dim() != 5 or t.shape[0] != g.planes or not t.is_contiguous():
                raise ValueError(f"layer tensor shape {tuple(t.shape)} does not match {g.name}")
            kind = "device" if t.is_cuda else ("pinned" if t.is_pinned() else "host")
            handles.append(self.runtime.register_memory(t.data_ptr(), t.numel() * t.element_size(), kind,
                                                        t.device.index if t.is_cuda else -1))
        self._layer_mems = np.asarray(handles, dtype=np.uint64)
        self._pool = (layers[0], int(handles[0]), layers[0].shape[1])
        return handles

    def targets_for(self, paths: Sequence[str]) -> list[int]:
        missing = sorted({p for p in paths if p not in self._targets})
        if missing:
            handles = self.runtime.open_batch(["file://" + p for p in missing])
            for p, h in zip(missing, handles):
                self._targets[p] = h
        return [self._targets[p] for p in paths]

    def warm_targets(self) -> int:
        """Open every ready segment file once (ticket cache warm-up)."""
        s = self.objects
        files = sorted({s.slot_path(i) for i in range(s.ready_slots)})
        self.targets_for(files)
        return len(files)

    # -- object queries -----------------------------------------------------
    def contains_prefix(self, keys: Sequence[bytes], all_ranks: bool = False) -> int:
        return self.objects.contains_prefix(list(keys), all_ranks)

    def drop(self, keys: Sequence[bytes]) -> int:
        return self.objects.release(list(keys))

    def scan(self) -> list[bytes]:
        return self.objects.recover()

    # -- paged IO -------------------------------------------------------------
    def _stream_ptr(self, stream) -> int:
        if self.backend != "nvme-gpu":
            return 0
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return s.cuda_stream

    def page_requests(self, placements: Sequence[tuple[str, int]], block_ids: np.ndarray,
                      layers: np.ndarray) -> tuple[np.ndarray, ...]:
        """(target handles, target offsets, memory offsets, lengths) in (chunk, layer, block, plane) order."""
        g = self.geometry
        if self.stored["transform"]:
            raise NotImplementedError("transformed stores submit through submit_paged (get_paged/put_paged)")
        if self._pool is None:
            raise RuntimeError("register_pool() first")
        nb = self._pool[2]
        n, bpc = block_ids.shape
        if bpc != g.blocks_per_chunk:
            raise ValueError(f"block table rows must hold {g.blocks_per_chunk} blocks")
        paths = [p for p, _ in placements]
        handles = np.asarray(self.targets_for(paths), dtype=np.uint64)
        base = np.asarray([o for _, o in placements], dtype=np.uint64)
        L = layers.astype(np.uint64)
        P = np.arange(g.planes, dtype=np.uint64)
        J = np.arange(bpc, dtype=np.uint64)
        pb = np.uint64(g.plane_block_bytes)
        tgt_off = (base[:, None, None, None] + L[None, :, None, None] * np.uint64(g.segment_bytes)
                   + J[None, None, :, None] * np.uint64(g.block_layer_bytes) + P[None, None, None, :] * pb)
        blk = block_ids.astype(np.uint64)
        mem_off = ((L[None, :, None, None] * np.uint64(g.planes) + P[None, None, None, :]) * np.uint64(nb)
                   + blk[:, None, :, None]) * pb
        shape = (n, L.size, bpc, g.planes)
        tgts = np.broadcast_to(handles[:, None, None, None], shape)
        lens = np.full(int(np.prod(shape)), g.plane_block_bytes, dtype=np.uint64)
        return (np.ascontiguousarray(tgts).reshape(-1), np.ascontiguousarray(tgt_off).reshape(-1),
                np.ascontiguousarray(mem_off).reshape(-1), lens)

    def _submit_retry(self, direction: str, tgts, tgt_off, mem_off, lens, stream) -> list[int]:
        ios: list[int] = []
        idx = np.arange(lens.size)
        mem = np.asarray([self._pool[1]], dtype=np.uint64)
        sptr = self._stream_ptr(stream)
        host = self.backend != "nvme-gpu"
        for attempt in range(self.max_retries):
            r = self.runtime.submit_arrays(direction, mem, mem_off[idx], tgts[idx], tgt_off[idx], lens[idx],
                                           sptr, host)
            if "runtime_submit_ms" in r:
                self.last_submit_profile = {k: v for k, v in r.items() if k.endswith("_ms") or k == "dp_commands"}
            if r["io"] is not None:
                ios.append(r["io"])
            rej = np.asarray(r["rejected"], dtype=np.int64)
            if rej.size == 0:
                return ios
            reasons = " ".join(r["reasons"])
            if "BUSY" not in reasons and "RESOURCE_EXHAUSTED" not in reasons:
                raise StoreIOError(f"{rej.size} request(s) rejected: {reasons}", idx[rej].tolist(), "rejected")
            idx = idx[rej]
            # Free queue leases / terminal-result budget: drain the oldest batch.
            if self._inflight:
                self._inflight.popleft().wait()
            elif ios:
                comp = NativeCompletion(self.runtime, ios)
                comp.wait()
                ios = []
            else:
                time.sleep(0.0005)
        raise StoreIOError("submit retries exhausted", idx.tolist(), "busy")

    def register_peer_pool(self, ptr: int, nbytes: int, device: int) -> int:
        """Register another GPU's whole KV pool (CUDA-IPC mapped) as a restore destination."""
        return self.runtime.register_memory(int(ptr), int(nbytes), "device", int(device))

    def restore_placements(self, placements, block_ids, chunk_mems=None, layers=None, stream=None, layer_mems=None,
                           chunk_layer_mems=None):
        """Restore chunks given by explicit (segment file path, payload offset) placements.

        ``chunk_mems[i]`` names the pool (this rank's or a peer's) chunk i lands in;
        ``layer_mems[l]`` instead names the per-layer tensor layer l lands in (a peer's
        per-layer caches, mapped through IPC); ``chunk_layer_mems[i, l]`` names layer
        l's tensor of the rank chunk i lands in (one submission for several ranks'
        per-layer caches: a placement named for several ranks is read once).
        Placements may belong to other ranks' namespaces (the files are opened here).
        """
        g = self.geometry
        block_ids = np.asarray(block_ids, dtype=np.int64).reshape(len(placements), g.blocks_per_chunk)
        layers = np.arange(g.num_layers) if layers is None else np.asarray(layers, dtype=np.int64).reshape(-1)
        cm = None if chunk_mems is None else np.asarray(chunk_mems, dtype=np.uint64)
        lm = None if layer_mems is None else np.asarray(layer_mems, dtype=np.uint64)
        clm = None if chunk_layer_mems is None else np.ascontiguousarray(chunk_layer_mems, dtype=np.uint64)
        ios, nbytes = self._submit_paged("read", placements, block_ids, layers, stream, chunk_mems=cm, layer_mems=lm,
                                         chunk_layer_mems=clm)
        comp = NativeCompletion(self.runtime, ios, nbytes=nbytes)
        self._track(comp)
        return comp

    def write_placements(self, placements, block_ids, chunk_mems=None, stream=None, layer_mems=None,
                         chunk_layer_mems=None) -> NativeCompletion:
        """Write all layers of chunks to explicit (segment file path, payload offset) placements.

        The slots must already be reserved (by this rank or by the rank that owns them);
        committing them is the caller's job. ``chunk_mems[i]`` names the pool the chunk is
        gathered from (a peer's pool is read over NVLink by the io kernel);
        ``chunk_layer_mems[i, l]`` instead names layer l's tensor of the rank chunk i is
        gathered from (per-layer caches, several ranks in one submission).
        """
        g = self.geometry
        block_ids = np.asarray(block_ids, dtype=np.int64).reshape(len(placements), g.blocks_per_chunk)
        cm = None if chunk_mems is None else np.asarray(chunk_mems, dtype=np.uint64)
        if stream is None and self.backend == "nvme-gpu":
            stream = torch.cuda.current_stream(self.device)
        lm = None if layer_mems is None else np.asarray(layer_mems, dtype=np.uint64)
        clm = None if chunk_layer_mems is None else np.ascontiguousarray(chunk_layer_mems, dtype=np.uint64)
        ios, nbytes = self._submit_paged("write", placements, block_ids, np.arange(g.num_layers), stream, chunk_mems=cm,
                                         layer_mems=lm, chunk_layer_mems=clm)
        comp = NativeCompletion(self.runtime, ios, nbytes=nbytes, kind="store")
        self._track(comp)
        return comp

    def _submit_paged(self, direction: str, placements, block_ids: np.ndarray, layers: np.ndarray, stream,
                      chunk_mems: np.ndarray | None = None, layer_mems: np.ndarray | None = None,
                      chunk_layer_mems: np.ndarray | None = None):
        """Paged requests generated natively (no per-request Python work); retried while leases are busy."""
        g = self.geometry
        handles = np.asarray(self.targets_for([p for p, _ in placements]), dtype=np.uint64)
        offsets = np.asarray([o for _, o in placements], dtype=np.uint64)
        st = self.stored
        geo = {"planes": g.planes, "plane_bytes": g.plane_block_bytes, "segment_bytes": st["segment_bytes"],
               "block_layer_bytes": g.block_layer_bytes, "num_blocks": int(self._pool[2]),
               "stored_plane_bytes": st["plane_bytes"], "stored_block_layer_bytes": st["block_layer_bytes"],
               "transform": st["transform"]}
        bt = np.ascontiguousarray(block_ids, dtype=np.int64)
        ly = np.ascontiguousarray(layers, dtype=np.int64)
        sptr = self._stream_ptr(stream)
        host = self.backend != "nvme-gpu"
        for _ in range(self.max_retries):
            none = np.zeros(0, dtype=np.uint64)
            if chunk_layer_mems is not None:
                r = self.runtime.submit_paged(direction, int(self._pool[1]), handles, offsets, bt, ly, geo, sptr, host,
                                              none, none, chunk_layer_mems)
            else:
                r = self.runtime.submit_paged(direction, int(self._pool[1]), handles, offsets, bt, ly, geo, sptr, host,
                                              self._layer_mems if layer_mems is None else layer_mems,
                                              chunk_mems if chunk_mems is not None else none)
            if not r["rejected"]:
                return [r["io"]], int(r["count"]) * g.plane_block_bytes
            reasons = " ".join(r["reasons"])
            if r["io"] is not None or ("BUSY" not in reasons and "RESOURCE_EXHAUSTED" not in reasons):
                if r["io"] is not None:
                    NativeCompletion(self.runtime, [r["io"]]).wait()
                raise StoreIOError(f"{len(r['rejected'])} request(s) rejected: {reasons}", r["rejected"], "rejected")
            metrics().add("submit_retries")
            if self._inflight:
                self._inflight.popleft().wait()
            else:
                time.sleep(0.0005)
        raise StoreIOError("submit retries exhausted", kind="busy")

    def get_paged(self, keys: Sequence[bytes], block_ids, layers=None, stream=None) -> NativeCompletion:
        """Restore chunks ``keys`` into pool blocks ``block_ids[i]`` for ``layers`` (default all)."""
        g = self.geometry
        block_ids = np.asarray(block_ids, dtype=np.int64).reshape(len(keys), g.blocks_per_chunk)
        layers = np.arange(g.num_layers) if layers is None else np.asarray(layers, dtype=np.int64).reshape(-1)
        placements = []
        for k in keys:
            p = self.objects.lookup(bytes(k))
            if p is None:
                raise StoreIOError(f"chunk {bytes(k).hex()} is not committed", kind="not_found")
            uri, off, _slot, _gen = p
            placements.append((uri[len("file://"):], off))
        with nvtx_range(f"tutti.restore|chunks={len(keys)}|layers={len(layers)}"):
            ios, nbytes = self._submit_paged("read", placements, block_ids, layers, stream)
        comp = NativeCompletion(self.runtime, ios, nbytes=nbytes)
        self._track(comp)
        return comp

    def reserve(self, keys: Sequence[bytes]):
        """Reserve slots for ``keys``, materialising more segment-file groups when the ready ones run out.

        Returns the object store's ``(accepted, rejected_count)``; accepted rows are
        ``(key, uri, offset, slot, generation)``.
        """
        keys = [bytes(k) for k in keys]
        accepted, rejected = self.objects.reserve(keys)
        if rejected:
            got = {bytes(a[0]) for a in accepted}
            rest = [k for k in keys if k not in got]
            self.layout.precreate_until(self.objects.ready_slots + len(rest))
            more, rejected = self.objects.reserve(rest)
            accepted = list(accepted) + list(more)
        return accepted, rejected

    def put_paged(self, keys: Sequence[bytes], block_ids, stream=None) -> NativeCompletion:
        """Persist all layers of chunks ``keys`` from pool blocks ``block_ids[i]``; commit on wait."""
        g = self.geometry
        keys = [bytes(k) for k in keys]
        block_ids = np.asarray(block_ids, dtype=np.int64).reshape(len(keys), g.blocks_per_chunk)
        fresh = [i for i, k in enumerate(keys) if not self.objects.contains(k)]
        if not fresh:
            return NativeCompletion(self.runtime, [])
        accepted, rejected = self.reserve([keys[i] for i in fresh])
        if rejected:
            self.objects.abort([a[0] for a in accepted])
            raise StoreIOError(f"{rejected} chunk(s) did not fit (capacity)", kind="capacity")
        # reserve() may return rows out of input order after growing: follow the input order
        by_key = {bytes(a[0]): a for a in accepted}
        accepted = [by_key[keys[i]] for i in fresh]
        placements = [(uri[len("file://"):], off) for (_k, uri, off, _s, _g) in accepted]
        wkeys = [a[0] for a in accepted]
        if self.backend == "nvme-gpu" and stream is None:
            # The gather reads the pool: order it after work queued on the current stream.
            stream = torch.cuda.current_stream(self.device)
        try:
            with nvtx_range(f"tutti.store|chunks={len(fresh)}"):
                ios, nbytes = self._submit_paged("write", placements, block_ids[fresh], np.arange(g.num_layers),
                                                 stream)
        except Exception:
            self.objects.abort(wkeys)
            raise
        comp = NativeCompletion(self.runtime, ios, on_success=lambda: self._commit(wkeys),
                                on_failure=lambda: self.objects.abort(wkeys), nbytes=nbytes, kind="store")
        self._track(comp)
        return comp

    def _commit(self, keys) -> None:
        """Payload durable on the drives first (a drive's write cache is written back), then the
        object store's commit (payload fdatasync, headers, their fdatasync)."""
        flush = getattr(self.runtime, "flush_devices", None)
        if flush is not None:
            flush()
        self.objects.commit(keys)

    def _track(self, comp: NativeCompletion) -> None:
        self._inflight.append(comp)
        while self._inflight and self._inflight[0].query() and len(self._inflight) > 64:
            self._inflight.popleft().wait()

    def wait_all(self) -> None:
        while self._inflight:
            self._inflight.popleft().wait()
