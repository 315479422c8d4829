"""Prefix index of the KV store: chained chunk keys and chunk residency.

Keys (fixed by the storage format; the GPU kernel ``tutti_b200.ops.prefix_hash``
computes the same bytes, and segment-file headers store them)::

    key_0 = blake2b(namespace || le64(t_0) .. le64(t_{C-1}), digest_size=16)
    key_i = blake2b(key_{i-1} || le64(tokens of chunk i),   digest_size=16)
    io_key = chunk_key(16) || le16(layer)

A trailing partial chunk has no key.

Residency is a table of ``_Rec`` records, one per chunk key the index knows.
A record is either PENDING (a write was planned and not yet settled: it takes
capacity, is never a hit and is never evicted) or RESIDENT. Each record keeps
its pin count, the epoch it was planned in and a recency stamp from a logical
clock that every hit advances. Three side structures keep the hot operations
away from full scans:

* ``_victims``: a min-heap of ``(stamp, key)`` for resident, unpinned
  records. Entries are invalidated lazily (a hit, a pin or a removal leaves
  the old entry behind; it is skipped when popped because its stamp no
  longer matches), and the heap is rebuilt when stale entries outnumber live
  ones. Choosing k victims costs O(k log n) whatever is pinned.
* ``_by_epoch``: pending keys bucketed by planning epoch, so reclaiming
  reservations that no rank ever settled visits only the expired buckets.
* counters of resident and pending records for the capacity check.

The class is single-threaded; callers serialise (the scheduler and each
worker engine own one index each).

Parity: the reference keeps the same key chain and the same residency rules
(plan reserves, confirm publishes, pins protect, pending never hits or is
evicted, LRU eviction inside plan_store only) in tutti/index/chunk_index.py:54-414;
this table-and-heap layout is this package's own.
"""
from __future__ import annotations

import hashlib
import heapq
import struct
from typing import Iterable, NamedTuple, Sequence

KEY_BYTES = 16
LAYER_BYTES = 2
IO_KEY_BYTES = KEY_BYTES + LAYER_BYTES

_PENDING = 1
_RESIDENT = 2


# -- key derivation ----------------------------------------------------------

def _token_bytes(tokens: Sequence[int]) -> bytes:
    """Little-endian uint64 encoding of token ids."""
    return struct.pack(f"<{len(tokens)}Q", *tokens)


def chunk_digest(parent: bytes, chunk: Sequence[int]) -> bytes:
    """Key of one chunk given its parent key (or the namespace for the first chunk)."""
    h = hashlib.blake2b(digest_size=KEY_BYTES)
    h.update(parent)
    h.update(_token_bytes(chunk))
    return h.digest()


def chunk_keys_for_tokens(tokens: Sequence[int], chunk_tokens: int, namespace: bytes = b"",
                          parent: bytes | None = None) -> list[bytes]:
    """Chained keys of every complete chunk of ``tokens``."""
    keys: list[bytes] = []
    prev = namespace if parent is None else parent
    whole = len(tokens) // chunk_tokens
    for c in range(whole):
        prev = chunk_digest(prev, tokens[c * chunk_tokens:(c + 1) * chunk_tokens])
        keys.append(prev)
    return keys


def derive_io_key(chunk_key: bytes, layer: int) -> bytes:
    """Object key of one layer of one chunk."""
    if not isinstance(chunk_key, (bytes, bytearray)) or len(chunk_key) != KEY_BYTES:
        raise ValueError(f"chunk key must be {KEY_BYTES} bytes")
    if isinstance(layer, bool) or not isinstance(layer, int) or not 0 <= layer < (1 << (8 * LAYER_BYTES)):
        raise ValueError(f"layer out of range: {layer!r}")
    return bytes(chunk_key) + struct.pack("<H", layer)


def decode_io_key(io_key: bytes) -> tuple[bytes, int]:
    """(chunk key, layer) of an object key (a bare chunk key decodes as layer 0)."""
    if not isinstance(io_key, (bytes, bytearray, memoryview)) or len(io_key) == 0:
        raise ValueError("io_key must be non-empty bytes")
    raw = bytes(io_key)
    return raw[:KEY_BYTES], int.from_bytes(raw[KEY_BYTES:], "little")


def _strict_io_key(io_key) -> bytes:
    if not isinstance(io_key, (bytes, bytearray)) or len(io_key) != IO_KEY_BYTES:
        raise ValueError(f"io_key must be {IO_KEY_BYTES} bytes")
    return bytes(io_key)


def chunk_key_of(io_key: bytes) -> bytes:
    return _strict_io_key(io_key)[:KEY_BYTES]


def layer_of(io_key: bytes) -> int:
    return struct.unpack("<H", _strict_io_key(io_key)[KEY_BYTES:])[0]


# -- residency ----------------------------------------------------------------

class StorePlan(NamedTuple):
    """Outcome of a write reservation: chunks to write, and chunks to drop first (coldest first)."""

    new_keys: list[bytes]
    evicted_keys: list[bytes]


class _Rec:
    __slots__ = ("state", "pins", "epoch", "stamp")

    def __init__(self, state: int, epoch: int, stamp: int):
        self.state = state
        self.pins = 0
        self.epoch = epoch
        self.stamp = stamp


class ChunkIndex:
    """Residency of chunk keys under a fixed capacity, with the key chain of one namespace."""

    def __init__(self, capacity: int, chunk_tokens: int, namespace: bytes = b""):
        if capacity <= 0:
            raise ValueError("capacity must be positive")
        if chunk_tokens <= 0:
            raise ValueError("chunk_tokens must be positive")
        if not isinstance(namespace, (bytes, bytearray)):
            raise ValueError("namespace must be bytes")
        self._capacity = int(capacity)
        self._chunk_tokens = int(chunk_tokens)
        self._namespace = bytes(namespace)
        self._recs: dict[bytes, _Rec] = {}
        self._victims: list[tuple[int, bytes]] = []
        self._by_epoch: dict[int, set[bytes]] = {}
        self._n_resident = 0
        self._n_pending = 0
        self._n_pinned = 0
        self._clock = 0
        self._epoch = 0

    # -- facts ------------------------------------------------------------------
    @property
    def capacity(self) -> int:
        return self._capacity

    @property
    def chunk_tokens(self) -> int:
        return self._chunk_tokens

    @property
    def namespace(self) -> bytes:
        return self._namespace

    @property
    def epoch(self) -> int:
        return self._epoch

    def stats(self) -> dict[str, int]:
        return {"capacity": self._capacity, "resident": self._n_resident, "pending": self._n_pending,
                "pinned": self._n_pinned, "epoch": self._epoch}

    def _state(self, key: bytes) -> int:
        rec = self._recs.get(key)
        return rec.state if rec is not None else 0

    def is_resident(self, key: bytes) -> bool:
        return self._state(key) == _RESIDENT

    def is_pending(self, key: bytes) -> bool:
        return self._state(key) == _PENDING

    def is_pinned(self, key: bytes) -> bool:
        rec = self._recs.get(key)
        return rec is not None and rec.pins > 0

    # -- recency and victims ------------------------------------------------------
    def _tick(self) -> int:
        self._clock += 1
        return self._clock

    def _offer(self, key: bytes, rec: _Rec) -> None:
        """Make a resident, unpinned record an eviction candidate at its current stamp."""
        heapq.heappush(self._victims, (rec.stamp, key))
        if len(self._victims) > 64 and len(self._victims) > 4 * max(1, self._n_resident):
            self._victims = [(r.stamp, k) for k, r in self._recs.items() if r.state == _RESIDENT and r.pins == 0]
            heapq.heapify(self._victims)

    def _touch(self, key: bytes, rec: _Rec) -> None:
        rec.stamp = self._tick()
        if rec.pins == 0:
            self._offer(key, rec)

    def _live_victim(self, stamp: int, key: bytes) -> bool:
        rec = self._recs.get(key)
        return rec is not None and rec.state == _RESIDENT and rec.pins == 0 and rec.stamp == stamp

    def _take_victims(self, count: int, spare: set[bytes]) -> list[bytes] | None:
        """The ``count`` coldest evictable keys outside ``spare``; None (heap unchanged) if too few."""
        taken: list[tuple[int, bytes]] = []
        skipped: list[tuple[int, bytes]] = []
        seen: set[bytes] = set()
        while len(taken) < count and self._victims:
            stamp, key = heapq.heappop(self._victims)
            if key in seen or not self._live_victim(stamp, key):
                continue  # stale or duplicate entry (a record is offered again on unpin): dropped for good
            seen.add(key)
            (skipped if key in spare else taken).append((stamp, key))
        for item in skipped:
            heapq.heappush(self._victims, item)
        if len(taken) < count:
            for item in taken:
                heapq.heappush(self._victims, item)
            return None
        return [k for _s, k in taken]

    def _drop(self, key: bytes) -> None:
        rec = self._recs.pop(key)
        if rec.state == _RESIDENT:
            self._n_resident -= 1
        else:
            self._n_pending -= 1
            bucket = self._by_epoch.get(rec.epoch)
            if bucket is not None:
                bucket.discard(key)
                if not bucket:
                    del self._by_epoch[rec.epoch]
        if rec.pins:
            self._n_pinned -= 1

    def _publish(self, key: bytes) -> None:
        """Make ``key`` resident as the most recent chunk (new or previously pending)."""
        rec = self._recs.get(key)
        if rec is None:
            rec = self._recs[key] = _Rec(_RESIDENT, self._epoch, self._tick())
            self._n_resident += 1
        elif rec.state == _PENDING:
            self._drop(key)
            rec = self._recs[key] = _Rec(_RESIDENT, self._epoch, self._tick())
            self._n_resident += 1
        else:
            rec.stamp = self._tick()
        if rec.pins == 0:
            self._offer(key, rec)

    # -- epochs -------------------------------------------------------------------
    def advance_epoch(self) -> int:
        self._epoch += 1
        return self._epoch

    def reclaim_stale_pending(self, max_age: int) -> list[bytes]:
        """Release reservations planned ``max_age`` or more epochs ago (nobody settled them)."""
        if max_age <= 0:
            return []
        horizon = self._epoch - max_age
        expired = [e for e in self._by_epoch if e <= horizon]
        freed: list[bytes] = []
        for e in sorted(expired):
            for key in sorted(self._by_epoch.get(e, ())):
                self._drop(key)
                freed.append(key)
        return freed

    # -- hashing and lookup ---------------------------------------------------------
    def hash_keys(self, token_ids: Sequence[int], start: int = 0, parent: bytes | None = None,
                  max_keys: int | None = None) -> tuple[list[bytes], bytes]:
        """Keys of the complete chunks of ``token_ids[start:]`` chained from ``parent``.

        ``parent`` is the key of the chunk that ends at ``start`` (the
        namespace when None), so a caller can hash a growing prompt
        incrementally. Returns the keys and the last key (the next parent).
        """
        if start < 0:
            raise ValueError("start must be non-negative")
        if max_keys is not None and max_keys <= 0:
            raise ValueError("max_keys must be positive")
        n = (len(token_ids) - start) // self._chunk_tokens if len(token_ids) > start else 0
        if max_keys is not None:
            n = min(n, max_keys)
        tail = self._namespace if parent is None else parent
        keys = chunk_keys_for_tokens(token_ids[start:start + n * self._chunk_tokens], self._chunk_tokens,
                                     parent=tail)
        return keys, (keys[-1] if keys else tail)

    def lookup_prefix_keys(self, keys: Sequence[bytes]) -> int:
        """Tokens covered by the longest run of resident keys from the start; hits become most recent."""
        hits = 0
        for key in keys:
            rec = self._recs.get(key)
            if rec is None or rec.state != _RESIDENT:
                break
            self._touch(key, rec)
            hits += 1
        return hits * self._chunk_tokens

    def lookup_prefix(self, token_ids: Sequence[int]) -> int:
        """Hash ``token_ids`` chunk by chunk and stop at the first chunk that is not resident."""
        prev = self._namespace
        hits = 0
        step = self._chunk_tokens
        for c in range(len(token_ids) // step):
            prev = chunk_digest(prev, token_ids[c * step:(c + 1) * step])
            rec = self._recs.get(prev)
            if rec is None or rec.state != _RESIDENT:
                break
            self._touch(prev, rec)
            hits += 1
        return hits * step

    def lookup_many(self, requests: Sequence[Sequence[int]], device=None) -> list[tuple[int, list[bytes]]]:
        """Prefix hits of many prompts at once: ``[(hit_tokens, keys)]`` per request.

        With ``device`` (a CUDA device), the keys of every request are hashed
        in one launch of the GPU prefix-hash kernel, which gives the same bytes
        as the host chain; otherwise they are hashed on the host.
        """
        if device is not None:
            from .. import ops

            all_keys = ops.prefix_hash(requests, self._chunk_tokens, namespace=self._namespace, device=device)
        else:
            all_keys = [chunk_keys_for_tokens(r, self._chunk_tokens, namespace=self._namespace) for r in requests]
        return [(self.lookup_prefix_keys(keys), keys) for keys in all_keys]

    # -- writes -----------------------------------------------------------------------
    def plan_store(self, keys: Iterable[bytes]) -> StorePlan | None:
        """Reserve capacity for a batch of chunks about to be written.

        Keys already resident need no write. If the free capacity does not
        cover the new keys, the coldest resident, unpinned keys outside the
        batch are evicted (the caller drops their data). Returns None and
        changes nothing when a key of the batch is already pending or the
        evictable keys do not cover the deficit.
        """
        batch: list[bytes] = []
        seen: set[bytes] = set()
        for k in keys:
            if k not in seen:
                seen.add(k)
                batch.append(k)
        if any(self._state(k) == _PENDING for k in batch):
            return None
        fresh = [k for k in batch if self._state(k) != _RESIDENT]
        free = self._capacity - self._n_resident - self._n_pending
        victims: list[bytes] = []
        if len(fresh) > free:
            got = self._take_victims(len(fresh) - free, seen)
            if got is None:
                return None
            victims = got
            for k in victims:
                self._drop(k)
        bucket = self._by_epoch.setdefault(self._epoch, set())
        for k in fresh:
            self._recs[k] = _Rec(_PENDING, self._epoch, 0)
            self._n_pending += 1
            bucket.add(k)
        return StorePlan(fresh, victims)

    def confirm_store(self, keys: Iterable[bytes], ok: bool = True) -> None:
        """Settle reservations: published as most recent on success, released on failure."""
        for k in keys:
            state = self._state(k)
            if ok:
                self._publish(k)
            elif state == _PENDING:
                self._drop(k)

    # -- protection ---------------------------------------------------------------------
    def pin(self, keys: Iterable[bytes]) -> None:
        """Protect resident keys from eviction (counted); any key not resident -> KeyError, nothing pinned."""
        batch = list(keys)
        absent = [k for k in batch if self._state(k) != _RESIDENT]
        if absent:
            raise KeyError(absent)
        for k in batch:
            rec = self._recs[k]
            if rec.pins == 0:
                self._n_pinned += 1
            rec.pins += 1

    def unpin(self, keys: Iterable[bytes]) -> None:
        """Release one pin per key; a key without pins -> KeyError, nothing released."""
        batch = list(keys)
        need: dict[bytes, int] = {}
        for k in batch:
            need[k] = need.get(k, 0) + 1
        short = [k for k, n in need.items() if k not in self._recs or self._recs[k].pins < n]
        if short:
            raise KeyError(short)
        for k in batch:
            rec = self._recs[k]
            rec.pins -= 1
            if rec.pins == 0:
                self._n_pinned -= 1
                if rec.state == _RESIDENT:
                    self._offer(k, rec)

    def mark_recent(self, keys: Iterable[bytes]) -> None:
        for k in keys:
            rec = self._recs.get(k)
            if rec is not None and rec.state == _RESIDENT:
                self._touch(k, rec)

    def restore(self, keys: Iterable[bytes]) -> None:
        """Cold start: publish keys recovered from the store, oldest first, while capacity lasts."""
        for k in keys:
            if self._state(k) == _RESIDENT:
                continue
            if self._n_resident + self._n_pending >= self._capacity:
                break
            self._publish(k)

    def forget(self, keys: Iterable[bytes]) -> list[bytes]:
        """Drop residency of unpinned keys whose data was lost; returns the keys dropped."""
        gone: list[bytes] = []
        for k in keys:
            rec = self._recs.get(k)
            if rec is not None and rec.state == _RESIDENT and rec.pins == 0:
                self._drop(k)
                gone.append(k)
        return gone
