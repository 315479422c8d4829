"""``tutti.storage.memory``: the in-process store (tutti_b200's), with Tutti's constructor names.

``MemoryKVStore(segment_bytes, num_chunks)`` as in Tutti (tutti_b200's names are
``chunk_bytes`` / ``capacity_chunks``); ``register_buffer`` also takes writable
host buffers (bytearray, memoryview, ctypes arrays), viewed in place.
"""
import torch

from tutti_b200.storage.memory import MemoryKVStore as _MemoryKVStore


class MemoryKVStore(_MemoryKVStore):
    def __init__(self, segment_bytes: int | None = None, num_chunks: int | None = None, *,
                 chunk_bytes: int | None = None, capacity_chunks: int | None = None):
        size = segment_bytes if segment_bytes is not None else chunk_bytes
        if size is None or int(size) <= 0:
            raise ValueError("segment_bytes must be a positive integer")
        count = num_chunks if num_chunks is not None else capacity_chunks
        super().__init__(int(size), int(count) if count is not None else 1 << 20)

    def register_buffer(self, buffer, granularity: int):
        if not isinstance(buffer, torch.Tensor):
            buffer = torch.frombuffer(memoryview(buffer).cast("B"), dtype=torch.uint8)
        return super().register_buffer(buffer, granularity)
