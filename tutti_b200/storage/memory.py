"""In-process KVStore: chunk bytes live in host memory.

The reference bases every store test on the same class
(tutti/storage/memory.py:24); it is also the engine's default store for
CPU-only runs. Buffers are torch tensors (any device); an entry
``(key, buffer_id, offset)`` moves ``chunk_bytes`` bytes.
"""
from __future__ import annotations

from collections import OrderedDict
from collections.abc import Iterable, Sequence

import torch

from .base import DoneCompletion, StoreIOError


class MemoryKVStore:
    def __init__(self, chunk_bytes: int, capacity_chunks: int = 1 << 20):
        self.chunk_bytes = int(chunk_bytes)
        self._capacity = int(capacity_chunks)
        self._data: OrderedDict[bytes, torch.Tensor] = OrderedDict()
        self._buffers: dict[int, torch.Tensor] = {}
        self._next = 1
        self._open = False

    @property
    def capacity_chunks(self) -> int:
        return self._capacity

    def open(self) -> None:
        self._open = True

    def close(self) -> None:
        self._open = False

    def register_buffer(self, buffer: torch.Tensor, granularity: int) -> int | None:
        if granularity != self.chunk_bytes:
            return None
        bid = self._next
        self._next += 1
        self._buffers[bid] = buffer.view(torch.uint8).reshape(-1)
        return bid

    def unregister_buffer(self, bid: int) -> None:
        self._buffers.pop(bid, None)

    def _view(self, bid: int, off: int) -> torch.Tensor:
        buf = self._buffers[bid]
        if off < 0 or off + self.chunk_bytes > buf.numel():
            raise StoreIOError(f"offset {off} out of buffer range")
        return buf[off:off + self.chunk_bytes]

    def put_batch(self, batch: Sequence[tuple[bytes, int, int]]):
        for key, bid, off in batch:
            if key in self._data:
                self._data.move_to_end(key)
                continue
            while len(self._data) >= self._capacity:
                self._data.popitem(last=False)
            self._data[bytes(key)] = self._view(bid, off).to("cpu", copy=True)
        return DoneCompletion()

    def get_batch(self, batch: Sequence[tuple[bytes, int, int]]):
        missing = [i for i, (k, _, _) in enumerate(batch) if bytes(k) not in self._data]
        if missing:
            return DoneCompletion(StoreIOError("keys not resident", missing, "not_found"))
        for key, bid, off in batch:
            self._view(bid, off).copy_(self._data[bytes(key)])
        return DoneCompletion()

    def contains(self, key: bytes) -> bool:
        return bytes(key) in self._data

    def drop(self, keys: Sequence[bytes]) -> None:
        for k in keys:
            self._data.pop(bytes(k), None)

    def scan(self) -> Iterable[bytes]:
        return iter(())
