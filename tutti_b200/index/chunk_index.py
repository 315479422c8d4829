"""Semantic index: chained chunk keys, residency, pins, pending writes, LRU.

Key derivation (fixed by the storage format; the GPU kernel
``tutti_b200.ops.prefix_hash`` computes the same bytes):
    key_0 = blake2b(namespace || le64(t_0) ... le64(t_{C-1}), digest_size=16)
    key_i = blake2b(key_{i-1} || le64(tokens of chunk i), digest_size=16)
A trailing partial chunk has no key. ``io_key = chunk_key(16) || le16(layer)``.

State per key: resident (participates in hits and LRU), pending (a write was
planned and not yet settled: occupies capacity, never hit, never evicted),
pin count (> 0 protects from eviction). Eviction happens only in
``plan_store``. Single-threaded; callers serialise.
Parity: reference tutti/index/chunk_index.py:54-414.
"""
from __future__ import annotations

import hashlib
import sys
from array import array
from collections import Counter, OrderedDict
from dataclasses import dataclass
from typing import Iterable, Sequence

KEY_BYTES = 16
LAYER_BYTES = 2
IO_KEY_BYTES = KEY_BYTES + LAYER_BYTES


def _le64(tokens: Sequence[int]) -> bytes:
    a = array("Q", tokens)
    if sys.byteorder != "little":
        a.byteswap()
    return a.tobytes()


def chunk_digest(parent: bytes, chunk: Sequence[int]) -> bytes:
    return hashlib.blake2b(parent + _le64(chunk), digest_size=KEY_BYTES).digest()


def chunk_keys_for_tokens(tokens: Sequence[int], chunk_tokens: int, namespace: bytes = b"",
                          parent: bytes | None = None) -> list[bytes]:
    """Chained keys of every complete chunk of ``tokens``."""
    p = namespace if parent is None else parent
    out = []
    for i in range(0, len(tokens) - chunk_tokens + 1, chunk_tokens):
        p = chunk_digest(p, tokens[i:i + chunk_tokens])
        out.append(p)
    return out


def derive_io_key(chunk_key: bytes, layer: int) -> bytes:
    if not isinstance(chunk_key, (bytes, bytearray)) or len(chunk_key) != KEY_BYTES:
        raise ValueError(f"chunk key must be {KEY_BYTES} bytes")
    if not isinstance(layer, int) or isinstance(layer, bool) or not 0 <= layer < (1 << (8 * LAYER_BYTES)):
        raise ValueError(f"layer out of range: {layer!r}")
    return bytes(chunk_key) + layer.to_bytes(LAYER_BYTES, "little")


def decode_io_key(io_key: bytes) -> tuple[bytes, int]:
    if not isinstance(io_key, (bytes, bytearray, memoryview)) or len(io_key) == 0:
        raise ValueError("io_key must be non-empty bytes")
    io_key = bytes(io_key)
    return io_key[:KEY_BYTES], int.from_bytes(io_key[KEY_BYTES:], "little")


def chunk_key_of(io_key: bytes) -> bytes:
    _check_io_key(io_key)
    return bytes(io_key[:KEY_BYTES])


def layer_of(io_key: bytes) -> int:
    _check_io_key(io_key)
    return int.from_bytes(io_key[KEY_BYTES:], "little")


def _check_io_key(io_key) -> None:
    if not isinstance(io_key, (bytes, bytearray)) or len(io_key) != IO_KEY_BYTES:
        raise ValueError(f"io_key must be {IO_KEY_BYTES} bytes")


@dataclass
class StorePlan:
    new_keys: list[bytes]
    evicted_keys: list[bytes]  # oldest first; the caller drops their data


class ChunkIndex:
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
        self._resident: OrderedDict[bytes, None] = OrderedDict()  # LRU: oldest first
        self._pending: dict[bytes, int] = {}  # key -> epoch planned
        self._pins: Counter[bytes] = Counter()
        self._epoch = 0

    # -- properties ---------------------------------------------------------
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
        return {"capacity": self._capacity, "resident": len(self._resident), "pending": len(self._pending),
                "pinned": len(self._pins), "epoch": self._epoch}

    def is_resident(self, key: bytes) -> bool:
        return key in self._resident

    def is_pinned(self, key: bytes) -> bool:
        return self._pins.get(key, 0) > 0

    def is_pending(self, key: bytes) -> bool:
        return key in self._pending

    # -- epochs ---------------------------------------------------------------
    def advance_epoch(self) -> int:
        self._epoch += 1
        return self._epoch

    def reclaim_stale_pending(self, max_age: int) -> list[bytes]:
        """Drop reservations older than ``max_age`` epochs (a rank that never settled)."""
        if max_age <= 0:
            return []
        cutoff = self._epoch - max_age
        stale = [k for k, e in self._pending.items() if e <= cutoff]
        for k in stale:
            del self._pending[k]
        return stale

    # -- hashing and lookup -------------------------------------------------
    def hash_keys(self, token_ids: Sequence[int], start: int = 0, parent: bytes | None = None,
                  max_keys: int | None = None) -> tuple[list[bytes], bytes]:
        """Fold tokens from ``start`` (earlier tokens are already in ``parent``) into keys."""
        if start < 0:
            raise ValueError("start must be non-negative")
        if max_keys is not None and max_keys <= 0:
            raise ValueError("max_keys must be positive")
        p = self._namespace if parent is None else parent
        step = self._chunk_tokens
        end = len(token_ids) - step + 1
        if max_keys is not None:
            end = min(end, start + max_keys * step)
        keys = []
        for i in range(start, end, step):
            p = chunk_digest(p, token_ids[i:i + step])
            keys.append(p)
        return keys, p

    def lookup_prefix(self, token_ids: Sequence[int]) -> int:
        """Tokens of the longest resident chunk prefix; hits refresh the LRU."""
        matched = 0
        p = self._namespace
        step = self._chunk_tokens
        for i in range(0, len(token_ids) - step + 1, step):
            p = chunk_digest(p, token_ids[i:i + step])
            if p not in self._resident:
                break
            self._resident.move_to_end(p)
            matched += step
        return matched

    def lookup_prefix_keys(self, keys: Sequence[bytes]) -> int:
        matched = 0
        for k in keys:
            if k not in self._resident:
                break
            self._resident.move_to_end(k)
            matched += self._chunk_tokens
        return matched

    # -- two-phase store ------------------------------------------------------
    def plan_store(self, keys: Iterable[bytes]) -> StorePlan | None:
        """Reserve capacity for a write batch, evicting LRU unpinned keys if needed.

        Returns None (and changes nothing) if any key is already pending or the
        deficit cannot be covered by evictable keys outside the batch.
        """
        batch = list(dict.fromkeys(keys))
        in_batch = set(batch)
        if any(k in self._pending for k in batch):
            return None
        new = [k for k in batch if k not in self._resident]
        deficit = len(new) - (self._capacity - len(self._resident) - len(self._pending))
        evicted: list[bytes] = []
        if deficit > 0:
            for k in self._resident:
                if len(evicted) == deficit:
                    break
                if k not in in_batch and self._pins.get(k, 0) == 0:
                    evicted.append(k)
            if len(evicted) < deficit:
                return None
            for k in evicted:
                del self._resident[k]
        for k in new:
            self._pending[k] = self._epoch
        return StorePlan(new_keys=new, evicted_keys=evicted)

    def confirm_store(self, keys: Iterable[bytes], ok: bool = True) -> None:
        """Settle a planned batch: resident (most recent) on success, else release capacity."""
        for k in keys:
            self._pending.pop(k, None)
            if ok:
                self._resident.pop(k, None)
                self._resident[k] = None

    # -- protection -----------------------------------------------------------
    def pin(self, keys: Iterable[bytes]) -> None:
        batch = list(keys)
        missing = [k for k in batch if k not in self._resident]
        if missing:
            raise KeyError(missing)
        for k in batch:
            self._pins[k] += 1

    def unpin(self, keys: Iterable[bytes]) -> None:
        batch = list(keys)
        missing = [k for k in batch if self._pins.get(k, 0) <= 0]
        if missing:
            raise KeyError(missing)
        for k in batch:
            self._pins[k] -= 1
            if self._pins[k] == 0:
                del self._pins[k]

    def mark_recent(self, keys: Iterable[bytes]) -> None:
        for k in keys:
            if k in self._resident:
                self._resident.move_to_end(k)

    def restore(self, keys: Iterable[bytes]) -> None:
        """Cold start: publish keys recovered from the store (oldest first), within capacity."""
        for k in keys:
            if len(self._resident) + len(self._pending) >= self._capacity:
                break
            self._resident[k] = None

    def forget(self, keys: Iterable[bytes]) -> list[bytes]:
        """Drop residency of unpinned keys (data was lost or invalidated); returns those dropped."""
        dropped = []
        for k in keys:
            if k in self._resident and self._pins.get(k, 0) == 0:
                del self._resident[k]
                dropped.append(k)
        return dropped
