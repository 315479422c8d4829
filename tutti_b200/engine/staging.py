"""Reusable staging memory for stores that move chunks through buffers (the staged path).

Each direction (restore, store) owns one allocation registered with the store
once and reused by every batch: a batch of ``n`` chunks uses the first
``n × chunk_bytes``. A larger batch replaces the allocation with one sized
for the next power of two chunks, and the old registration is dropped.
Before the buffer is handed to the next batch, the previous batch must be
done with it. Two things are waited for: the device work it queued (an event
recorded at release) and, for stores, the store's completion of that batch,
because a store may read the buffer until its put completes.
Parity: reference tutti/engine/staging.py:8-120 (RingWindow: staging slots
rotated across batches, reuse gated by events).
"""
from __future__ import annotations

import contextlib
import logging
import threading

import torch

LOG = logging.getLogger("tutti_b200.engine")


class StagingBuffer:
    def __init__(self, store, chunk_bytes: int, device: torch.device):
        self.store = store
        self.chunk_bytes = int(chunk_bytes)
        self.device = device
        self._lock = threading.Lock()
        self._buf: torch.Tensor | None = None
        self._bid: int | None = None
        self._cap = 0
        self._event: torch.cuda.Event | None = None
        self._pending = None
        self.allocations = 0  # registrations made so far (grows only with the largest batch)

    @property
    def capacity_chunks(self) -> int:
        return self._cap

    def _settle_previous(self) -> None:
        if self._event is not None:
            self._event.synchronize()
            self._event = None
        if self._pending is not None:
            pending, self._pending = self._pending, None
            try:
                pending.wait()
            except Exception as e:  # noqa: BLE001 - the batch's owner handles (and has been told of) it
                LOG.warning("staged store batch failed: %s", e)

    def _grow(self, nchunks: int) -> None:
        self._drop_registration()
        cap = 1 << max(0, (nchunks - 1).bit_length())
        self._buf = torch.empty(cap * self.chunk_bytes, dtype=torch.uint8, device=self.device)
        bid = self.store.register_buffer(self._buf, self.chunk_bytes)
        if bid is None:
            self._buf = None
            raise RuntimeError("store refused the staging buffer")
        self._bid, self._cap = bid, cap
        self.allocations += 1

    def _drop_registration(self) -> None:
        if self._bid is not None and hasattr(self.store, "unregister_buffer"):
            self.store.unregister_buffer(self._bid)
        self._buf, self._bid, self._cap = None, None, 0

    @contextlib.contextmanager
    def use(self, nchunks: int, stream: torch.cuda.Stream | None = None):
        """Yields ``(view, buffer_id)`` for ``nchunks`` chunks; set ``holder["pending"]`` to gate reuse on it."""
        with self._lock:
            self._settle_previous()
            if self._cap < nchunks:
                self._grow(nchunks)
            holder = {"pending": None}
            try:
                yield self._buf[: nchunks * self.chunk_bytes], self._bid, holder
            finally:
                if self._buf is not None and self._buf.is_cuda:
                    ev = torch.cuda.Event()
                    ev.record(stream if stream is not None else torch.cuda.current_stream(self.device))
                    self._event = ev
                self._pending = holder["pending"]

    def close(self) -> None:
        with self._lock:
            self._settle_previous()
            self._drop_registration()
