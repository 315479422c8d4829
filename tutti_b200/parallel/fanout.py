"""Multi-GPU restore: drive-affine reads fanned out to TP peers over NVLink.

An NVMe drive hangs off one GPU's PCIe switch, while every TP rank needs its
own KV-head slice of each chunk. The drive-affine GPU reads the chunks stored
on its drives for *all* ranks and its fused io kernel stores each rank's
slice straight into that rank's paged pool (CUDA-IPC-mapped peer pointers,
P2P stores over NVLink 5/NVSwitch): no staging copy on the peer, no separate
scatter kernel, no NCCL all-gather. Replicated caches (an MLA latent cache is
identical on every TP rank) are read once and stored to every rank's pool by
the same kernel (replica groups). Each rank then orders its own later work
after every rank's share on the device: a ReadyBoard flag that each rank
raises behind its io kernel and that the consumer's stream waits on (bounded),
with no host round trip; ``FanoutRestorer.barrier`` is the host-side form.

Control plane: pool IPC handles and per-rank placements are exchanged with
``torch.distributed`` object collectives (no data crosses it).
Parity: reference tutti/storage/tutti_nvme/replica_direct.py:43-1190 (owner =
le64(key[:8]) % group, owner reads, consumers pull pages through IPC with
replica_page_scatter_kernel) and the replica-sharded IO design notes; here the
owner pushes inside the io kernel instead of consumers pulling afterwards.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np
import torch
import torch.distributed as dist

from .. import ops


def owner_of(key: bytes, group_size: int) -> int:
    """Replica owner of a chunk: its first 8 key bytes, little-endian, modulo the group."""
    return int.from_bytes(bytes(key[:8]), "little") % group_size


class ReadyBoard:
    """Device-side ordering between the ranks of a group.

    Every rank holds a ``[slots, world]`` board of 64-bit words in its own HBM,
    mapped into every peer through CUDA IPC. ``signal(slot, value)`` stores
    ``value`` into this rank's column of ``slot`` on every board, on a stream,
    behind that stream's earlier work (a system-scope fence first, so the io
    kernel's NVLink stores to the peers are visible before the flag).
    ``wait(slot, value)`` makes a stream wait until every rank's word of
    ``slot`` on this rank's board reached ``value``: one thread of one CTA
    polls, bounded by a deadline; past it the stream continues and
    ``failed(ticket)`` reports which ranks were missing. Values grow
    monotonically (an epoch per restore), so a slot is reused without a reset.
    """

    def __init__(self, device: int, group=None, slots: int = 64, status_words: int = 1024):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.slots = slots
        self.device = device
        self.board = torch.zeros(slots, self.world, dtype=torch.int64, device=device)
        handle, offset, _ = ops.ipc_export(self.board)
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, (handle, offset, device), group=group)
        self._opened: list[int] = []
        bases = []
        for r, (h, off, devi) in enumerate(everyone):
            if r == self.rank:
                bases.append(self.board.data_ptr())
            else:
                ops.enable_peer_access(device, devi)
                base = ops.ipc_open(h, device)
                self._opened.append(base)
                bases.append(base + off)
        # targets[s, r]: this rank's word of slot s on rank r's board
        t = [[bases[r] + 8 * (s * self.world + self.rank) for r in range(self.world)] for s in range(slots)]
        self._targets = torch.tensor(t, dtype=torch.int64, device=device)
        self._status = torch.zeros(status_words, dtype=torch.int32).pin_memory()
        self._next_status = 0

    def signal(self, slot: int, value: int, stream: torch.cuda.Stream | None = None) -> None:
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            ops.ready_signal(self._targets[slot], value)

    def wait(self, slot: int, value: int, stream: torch.cuda.Stream | None = None, timeout_s: float = 10.0) -> int:
        """Enqueue the wait; returns a ticket for ``failed`` (read once the stream passed the wait)."""
        ticket = self._next_status
        self._next_status = (self._next_status + 1) % self._status.numel()
        self._status[ticket] = -1
        words = self.board.data_ptr() + 8 * slot * self.world
        with torch.cuda.stream(stream or torch.cuda.current_stream(self.device)):
            ops.ready_wait(words, self.world, value, int(timeout_s * 1e9), self._status[ticket:ticket + 1])
        return ticket

    def passed(self, ticket: int) -> bool:
        """True once the stream ran the wait (its outcome is then readable with ``failed``)."""
        return (int(self._status[ticket]) & 0xFFFFFFFF) != 0xFFFFFFFF

    def failed(self, ticket: int) -> list[int]:
        """Ranks the wait gave up on (empty: all arrived); valid after the stream passed the wait."""
        v = int(self._status[ticket]) & 0xFFFFFFFF
        if v == 0xFFFFFFFF:
            raise RuntimeError("the wait has not run yet")
        return [r for r in range(min(self.world, 31)) if v & (1 << r)] + ([31] if v & (1 << 31) else [])

    def close(self) -> None:
        for p in self._opened:
            ops.ipc_close(p, self.device)
        self._opened.clear()


class PeerPools:
    """Every rank's KV pool, mapped into this process through CUDA IPC."""

    def __init__(self, pool: torch.Tensor, group=None):
        self.pool = pool
        self.device = pool.device.index
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        handle, offset, _size = ops.ipc_export(pool)
        mine = (handle, offset, self.device, pool.numel() * pool.element_size())
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.ptrs: list[int] = []
        self.devices: list[int] = []
        self.nbytes: list[int] = []
        self._opened: list[int] = []
        for r, (h, off, devi, nb) in enumerate(everyone):
            if r == self.rank:
                self.ptrs.append(pool.data_ptr())
            else:
                ops.enable_peer_access(self.device, devi)
                base = ops.ipc_open(h, self.device)
                self._opened.append(base)
                self.ptrs.append(base + off)
            self.devices.append(devi)
            self.nbytes.append(nb)

    def close(self) -> None:
        for p in self._opened:
            ops.ipc_close(p, self.device)
        self._opened.clear()


class PeerLayers:
    """Every rank's per-layer KV tensors (one allocation per layer, as vLLM keeps
    them), mapped into this process through CUDA IPC: ``ptrs[r][l]``."""

    def __init__(self, layers: Sequence[torch.Tensor], group=None):
        self.layers = list(layers)
        self.device = self.layers[0].device.index
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        mine = []
        for t in self.layers:
            h, off, _size = ops.ipc_export(t)
            mine.append((h, off, t.numel() * t.element_size()))
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, (self.device, mine), group=group)
        self.ptrs: list[list[int]] = []
        self.nbytes: list[list[int]] = []
        self.devices: list[int] = []
        self._opened: list[int] = []
        for r, (devi, entries) in enumerate(everyone):
            self.devices.append(devi)
            self.nbytes.append([nb for _h, _o, nb in entries])
            if r == self.rank:
                self.ptrs.append([t.data_ptr() for t in self.layers])
                continue
            ops.enable_peer_access(self.device, devi)
            row = []
            for h, off, _nb in entries:
                base = ops.ipc_open(h, self.device)
                self._opened.append(base)
                row.append(base + off)
            self.ptrs.append(row)

    def close(self) -> None:
        for p in self._opened:
            ops.ipc_close(p, self.device)
        self._opened.clear()


@dataclass
class FaninBatch:
    """One step's saves in flight through the drive-affine GPUs (``FanoutRestorer.store_begin``)."""

    batch_id: int
    keys: list = field(default_factory=list)  # this rank's reserved keys (committed or aborted together)
    comp: object = None  # this GPU's writes (None: it had nothing to write)
    ticket: int | None = None  # the device wait for every rank's forward, on the io stream
    reuse_tickets: list = field(default_factory=list)  # device waits of forwards that reuse the blocks
    error: str = ""
    committed: bool | None = None

    def local_state(self, board, blocking: bool = False) -> str:
        """"pending", "ok" or "fail" on this rank."""
        if self.error:
            return "fail"
        if self.comp is not None:
            if not blocking and not self.comp.query():
                return "pending"
            try:
                self.comp.wait()
            except Exception as e:  # noqa: BLE001
                self.error = str(e)
                return "fail"
        for t in ([self.ticket] if self.ticket is not None else []) + list(self.reuse_tickets):
            if not board.passed(t):
                if not blocking:
                    return "pending"
                torch.cuda.synchronize()
            if board.failed(t):
                self.error = "a device wait gave up"
                return "fail"
        return "ok"


@dataclass
class RestoreItem:
    """Restore chunk ``key`` into rank ``rank``'s pool blocks ``block_ids``.

    ``source`` is the rank whose namespace holds the chunk: ``rank`` itself for a
    TP-sliced cache, the replica owner for a cache that is identical on every
    rank (all ranks' items of one key then share one read).
    """

    rank: int
    key: bytes
    block_ids: Sequence[int]
    source: int | None = None

    @property
    def src(self) -> int:
        return self.rank if self.source is None else self.source


class FanoutRestorer:
    """Restores (and stores) chunks for all ranks through the drives this GPU owns (drive-affine)."""

    def __init__(self, store, peers, group=None):
        self.kv = store
        self.peers = peers
        self.group = group
        if isinstance(peers, PeerLayers):
            # per-layer caches: layer l of rank r lands in layer_mems[r][l]
            self.mems = None
            self.layer_mems = []
            for r in range(peers.world):
                if r == peers.rank:
                    self.layer_mems.append(np.asarray(store._layer_mems, dtype=np.uint64))
                else:
                    self.layer_mems.append(np.asarray([store.register_peer_pool(p, nb, peers.devices[r])
                                                       for p, nb in zip(peers.ptrs[r], peers.nbytes[r])],
                                                      dtype=np.uint64))
        else:
            self.layer_mems = None
            self.mems = [store._pool[1] if r == peers.rank else store.register_peer_pool(p, peers.nbytes[r],
                                                                                        peers.devices[r])
                         for r, p in enumerate(peers.ptrs)]

    def placements(self, keys_by_rank: dict[int, Sequence[bytes]]) -> dict[tuple[int, bytes], tuple[str, int, int]]:
        """Every rank looks up its own chunks; the (path, offset, slot) map is shared by all."""
        mine = {}
        for k in keys_by_rank.get(self.peers.rank, []):
            p = self.kv.objects.lookup(bytes(k))
            if p is not None:
                uri, off, slot, _gen = p
                mine[(self.peers.rank, bytes(k))] = (uri[len("file://"):], off, slot)
        allmaps: list = [None] * self.peers.world
        dist.all_gather_object(allmaps, mine, group=self.group)
        out = {}
        for m in allmaps:
            out.update(m)
        return out

    def restore(self, items: Sequence[RestoreItem], n_drives: int, affine_gpus: Sequence[int],
                layers=None, stream=None, placements=None):
        """Submit this GPU's share: items whose chunk lives on a drive this GPU is affine to.

        Drive d (= slot % n_drives) belongs to GPU ``affine_gpus[d % len(affine_gpus)]``.
        Returns this rank's completion (None if it owns no drive); call ``barrier()`` after
        waiting so peers see the stores.
        """
        pl = placements if placements is not None else self.placements(
            {r: sorted({bytes(it.key) for it in items if it.src == r}) for r in range(self.peers.world)})
        todo, ranks, blocks = [], [], []
        for it in items:
            p = pl.get((it.src, bytes(it.key)))
            if p is None:
                raise KeyError(f"rank {it.src} has no committed chunk {bytes(it.key).hex()}")
            path, off, slot = p
            if affine_gpus[(slot % n_drives) % len(affine_gpus)] != self.peers.rank:
                continue
            todo.append((path, off))
            ranks.append(it.rank)
            blocks.append(list(it.block_ids))
        if not todo:
            return None
        if self.layer_mems is not None:
            # one submission for every destination rank: row i names the per-layer caches of
            # the rank item i lands in; a placement named for several ranks (a replicated
            # cache) becomes one read stored into each of them
            clm = np.stack([self.layer_mems[r] for r in ranks])
            return self.kv.restore_placements(todo, np.asarray(blocks, dtype=np.int64), layers=layers, stream=stream,
                                              chunk_layer_mems=clm)
        mems = [self.mems[r] for r in ranks]
        return self.kv.restore_placements(todo, np.asarray(blocks, dtype=np.int64), np.asarray(mems, np.uint64),
                                             layers=layers, stream=stream)

    def store(self, items: Sequence[RestoreItem], n_drives: int, affine_gpus: Sequence[int],
              stream=None) -> int:
        """Persist every rank's chunks through the drive-affine GPUs (gather over NVLink).

        Collective over the group. Each rank reserves slots for its own new chunks in its
        own namespace; the GPU affine to a slot's drive gathers the chunk's blocks from the
        owner's pool (P2P loads inside the io kernel) and writes them; once every rank's
        writes have completed, each rank commits its own chunks (or aborts them all if
        any write failed anywhere). Returns how many chunks this rank committed.
        """
        me = self.peers.rank
        objects = self.kv.objects
        mine = [it for it in items if it.rank == me and not objects.contains(bytes(it.key))]
        reserved, err = {}, ""
        if mine:
            reserve = getattr(self.kv, "reserve", objects.reserve)  # the store grows its files on demand
            accepted, rejected = reserve([bytes(it.key) for it in mine])
            for k, uri, off, slot, _gen in accepted:
                reserved[(me, bytes(k))] = (uri[len("file://"):], off, slot)
            if rejected:
                err = f"rank {me}: {rejected} chunk(s) did not fit"
        # the owners' pools must hold the blocks before any GPU gathers them
        if torch.cuda.is_available():
            torch.cuda.current_stream().synchronize()
        allmaps: list = [None] * self.peers.world
        dist.all_gather_object(allmaps, (reserved, err), group=self.group)
        placements, errors = {}, [e for _, e in allmaps if e]
        for m, _ in allmaps:
            placements.update(m)
        ok = not errors
        if ok:
            todo, ranks, blocks = [], [], []
            for it in items:
                p = placements.get((it.rank, bytes(it.key)))
                if p is None:
                    continue  # already stored
                path, off, slot = p
                if affine_gpus[(slot % n_drives) % len(affine_gpus)] != me:
                    continue
                todo.append((path, off))
                ranks.append(it.rank)
                blocks.append(list(it.block_ids))
            try:
                if todo and self.layer_mems is not None:
                    self.kv.write_placements(todo, np.asarray(blocks, dtype=np.int64), stream=stream,
                                             chunk_layer_mems=np.stack([self.layer_mems[r] for r in ranks])).wait()
                elif todo:
                    self.kv.write_placements(todo, np.asarray(blocks, dtype=np.int64),
                                             np.asarray([self.mems[r] for r in ranks], np.uint64), stream=stream).wait()
                # this GPU's drives hold other ranks' chunks too: durable before anyone commits
                flush = getattr(getattr(self.kv, "runtime", None), "flush_devices", None)
                if flush is not None:
                    flush()
            except Exception as e:  # noqa: BLE001  (reported through the collective below)
                errors.append(f"rank {me}: {e}")
                ok = False
        flags: list = [None] * self.peers.world
        dist.all_gather_object(flags, ok, group=self.group)
        keys = [k for (r, k) in reserved]
        if all(flags):
            objects.commit(keys)
            return len(keys)
        if keys:
            objects.abort(keys)
        if errors:
            raise RuntimeError("; ".join(errors))
        raise RuntimeError("a peer's drive-affine write failed; this rank's chunks were aborted")

    # -- asynchronous fan-in stores (the vLLM worker's saves under replica_io) -------------
    def store_begin(self, batch_id: int, items: Sequence[RestoreItem], mine: Sequence[bytes], n_drives: int,
                    affine_gpus: Sequence[int], board, stream=None) -> "FaninBatch":
        """Start persisting ``items`` through the drive-affine GPUs without waiting for the writes.

        Collective over the group, called by every rank for the same batch in the same
        order. This rank reserves ``mine`` (its own new keys) in its namespace and the
        reservations are exchanged; on ``stream`` this GPU then waits on the device until
        every rank raised ``board`` slot 0 to ``batch_id`` (its forward wrote the blocks),
        gathers the blocks of the chunks on its affine drives from their owners' caches
        (P2P loads in the io kernel) and writes them, and raises slot 1 to ``batch_id``
        behind the writes. Commits are decided later by ``store_harvest``.
        """
        me = self.peers.rank
        objects = self.kv.objects
        reserved, err = {}, ""
        mine = [bytes(k) for k in mine if not objects.contains(bytes(k))]  # stored by an earlier batch
        if mine:
            reserve = getattr(self.kv, "reserve", objects.reserve)
            accepted, rejected = reserve(mine)
            for k, uri, off, slot, _gen in accepted:
                reserved[(me, bytes(k))] = (uri[len("file://"):], off, slot)
            if rejected:
                err = f"rank {me}: {rejected} chunk(s) did not fit"
        allmaps: list = [None] * self.peers.world
        dist.all_gather_object(allmaps, (reserved, err), group=self.group)
        placements, errors = {}, [e for _, e in allmaps if e]
        for m, _ in allmaps:
            placements.update(m)
        batch = FaninBatch(batch_id, keys=[k for (_r, k) in reserved], error="; ".join(errors))
        if errors:
            board.signal(1, batch_id, stream)  # nothing will be written: no rank waits on this GPU
            return batch
        todo, ranks, blocks = [], [], []
        for it in items:
            p = placements.get((it.rank, bytes(it.key)))
            if p is None:
                continue  # already stored by its rank
            path, off, slot = p
            if affine_gpus[(slot % n_drives) % len(affine_gpus)] != me:
                continue
            todo.append((path, off))
            ranks.append(it.rank)
            blocks.append(list(it.block_ids))
        batch.ticket = board.wait(0, batch_id, stream)  # every rank's forward of this batch is done
        try:
            if todo and self.layer_mems is not None:
                batch.comp = self.kv.write_placements(todo, np.asarray(blocks, dtype=np.int64), stream=stream,
                                                      chunk_layer_mems=np.stack([self.layer_mems[r] for r in ranks]))
            elif todo:
                batch.comp = self.kv.write_placements(todo, np.asarray(blocks, dtype=np.int64),
                                                      np.asarray([self.mems[r] for r in ranks], np.uint64),
                                                      stream=stream)
        except Exception as e:  # noqa: BLE001 - reported through store_harvest
            batch.error = f"rank {me}: {e}"
        board.signal(1, batch_id, stream)
        return batch

    def store_harvest(self, batches: Sequence["FaninBatch"], board, blocking: bool = False) -> list["FaninBatch"]:
        """Decide the batches every rank has finished: commit each rank's own keys, or abort them.

        Collective over the group (every rank calls it at the same point with the same
        batch ids). A batch is finished on this rank when its writes completed and every
        device wait registered on it (before the writes, and ``reuse_tickets`` of forwards
        that reuse its blocks) has run; it fails if a write failed or a wait gave up (a
        block may have changed while it was gathered). Returns the batches decided now,
        with ``committed`` set on each.
        """
        flushed = False
        local: dict[int, str] = {}
        for b in batches:
            state = b.local_state(board, blocking)
            if state == "ok" and b.comp is not None and not flushed:
                flush = getattr(getattr(self.kv, "runtime", None), "flush_devices", None)
                try:
                    if flush is not None:
                        flush()  # this GPU's drives hold other ranks' chunks too: durable first
                except Exception as e:  # noqa: BLE001
                    b.error = b.error or f"rank {self.peers.rank}: flush: {e}"
                    state = "fail"
                flushed = True
            local[b.batch_id] = state
        states: list = [None] * self.peers.world
        dist.all_gather_object(states, local, group=self.group)
        decided = []
        for b in batches:
            seen = [st.get(b.batch_id, "pending") for st in states]
            if "pending" in seen:
                continue
            b.committed = all(x == "ok" for x in seen)
            if b.keys:
                (self.kv.objects.commit if b.committed else self.kv.objects.abort)(b.keys)
            decided.append(b)
        return decided

    def barrier(self) -> None:
        """Orders every rank after all ranks' restores (their kernels completed before this)."""
        if torch.cuda.is_available():
            torch.cuda.current_stream().synchronize()
        dist.barrier(group=self.group)


class FanoutLayerPlan:
    """Layer-by-layer drive-affine restore of one batch for every rank, ordered on the device.

    The placements are gathered here, on the calling thread (a collective of the
    group: every rank builds its plans in the same order). A feeder thread then
    submits, layer by layer, this GPU's share of every rank's chunks (at most
    ``window`` layers in flight) and raises the layer's flag on the ReadyBoard
    behind it on the IO stream, also when this GPU has nothing to read for the
    layer. ``wait_layer(l)`` makes the current stream wait until every rank raised
    layer l's flag for this plan's epoch; ``finish`` settles the submissions and
    reports ranks that never raised a flag.
    """

    def __init__(self, fan: FanoutRestorer, board: ReadyBoard, items: Sequence[RestoreItem], n_drives: int,
                 affine_gpus: Sequence[int], layers: Sequence[int], io_stream: torch.cuda.Stream, epoch: int,
                 window: int = 4, timeout_s: float = 30.0):
        import threading

        world = fan.peers.world
        self.fan, self.board, self.items = fan, board, list(items)
        self.n_drives, self.affine = n_drives, list(affine_gpus)
        self.layers, self.io_stream, self.epoch = list(layers), io_stream, epoch
        self.window, self.timeout_s = max(1, window), timeout_s
        self.placements = fan.placements({r: sorted({bytes(it.key) for it in items if it.src == r})
                                          for r in range(world)})
        self._comps: list = []
        self._submitted = 0
        self._tickets: list[int] = []
        self._error: BaseException | None = None
        self._cv = threading.Condition()
        self._thread = threading.Thread(target=self._feed, name="tutti-fanout-feeder", daemon=True)
        self._thread.start()

    def _feed(self) -> None:
        try:
            torch.cuda.set_device(self.board.device)
            for li, layer in enumerate(self.layers):
                if li >= self.window and self._comps[li - self.window] is not None:
                    self._comps[li - self.window].wait()
                comp = self.fan.restore(self.items, self.n_drives, self.affine, layers=[layer],
                                        stream=self.io_stream, placements=self.placements)
                self.board.signal(layer % self.board.slots, self.epoch, self.io_stream)
                with self._cv:
                    self._comps.append(comp)
                    self._submitted = li + 1
                    self._cv.notify_all()
        except BaseException as e:  # noqa: BLE001 - surfaced by wait_layer / finish
            # the peers' layer waits must not run into their deadlines: raise the
            # flags of the layers not submitted; the failure reaches every rank
            # through finish() and the TP failure consensus, not through the flags
            try:
                for layer in self.layers[len(self._comps):]:
                    self.board.signal(layer % self.board.slots, self.epoch, self.io_stream)
            except Exception:  # noqa: BLE001 - the original error is the one to report
                pass
            with self._cv:
                self._error = e
                self._cv.notify_all()

    def wait_layer(self, layer: int) -> None:
        li = self.layers.index(layer)
        with self._cv:
            while self._submitted <= li and self._error is None:
                self._cv.wait(timeout=self.timeout_s)
        # every rank's share of this layer, including the ones this GPU did not read
        self._tickets.append(self.board.wait(layer % self.board.slots, self.epoch, torch.cuda.current_stream(),
                                             self.timeout_s))

    def finish(self) -> None:
        from ..engine.completion import LoadGateError

        self._thread.join(timeout=self.timeout_s * len(self.layers))
        err = self._error
        for c in self._comps:
            if c is None:
                continue
            try:
                c.wait()
            except Exception as e:  # noqa: BLE001
                err = err or e
        torch.cuda.current_stream().synchronize()
        missing = sorted({r for t in self._tickets for r in self.board.failed(t)})
        if err is not None or missing:
            why = str(err) if err is not None else f"ranks {missing} never signalled"
            raise LoadGateError(f"fan-out restore failed: {why}")  # no chunk list: every chunk counts as failed

    def abort(self) -> None:
        try:
            self.finish()
        except Exception:  # noqa: BLE001
            pass

    def read_ms(self):
        return None
