"""Python view of the native segment-file object store.

One chunk (``chunk_tokens`` tokens, all layers of this rank's KV slice) is one
object in one slot of a fixed-size segment file; slots rotate over the backing
mounts (``slot % N``) and every payload starts ``segment_header_bytes`` into
its slot so it is 16 KiB-aligned on the device.
Parity: reference tutti/storage/tutti_nvme/object_layout.py:43-531
(defaults 2048 slots per file and a 128 KiB slot prefix, the geometry
fingerprint, background file-group precreate with a free-space guard).
"""
from __future__ import annotations

import os
import shutil
import threading
from pathlib import Path

from .._native import core

DEFAULT_SEGMENT_FILE_SLOTS = 2048
DEFAULT_SEGMENT_HEADER_BYTES = 128 * 1024
DEFAULT_PRECREATE_MIN_FREE_BYTES = 32 * 1024 ** 3


def layout_fingerprint(namespace: bytes, segment_file_slots: int, segment_header_bytes: int) -> bytes:
    """Namespace plus segment-file geometry: a change of either is another pool."""
    tag = (b"segment-files-rotating-v4-slots:" + str(int(segment_file_slots)).encode() + b"-header:" +
           str(int(segment_header_bytes)).encode())
    return (namespace or b"") + b"\0" + tag


class ObjectLayout:
    def __init__(self, root: str | os.PathLike, *, segment_bytes: int, segment_count: int,
                 capacity_chunks: int, mounts: list[str] | None = None, namespace: bytes = b"",
                 rank: int = 0, rank_count: int = 1,
                 segment_file_slots: int = DEFAULT_SEGMENT_FILE_SLOTS,
                 segment_header_bytes: int = DEFAULT_SEGMENT_HEADER_BYTES,
                 materialize: str = "zeros", read_only: bool = False,
                 precreate_min_free_bytes: int | None = None):
        self.root = Path(root)
        self.mounts = [str(m) for m in (mounts or [self.root])]
        self.segment_bytes = int(segment_bytes)
        self.segment_count = int(segment_count)
        self.capacity_chunks = int(capacity_chunks)
        self.namespace = namespace
        self.rank = rank
        self.rank_count = rank_count
        self.segment_file_slots = int(segment_file_slots)
        self.segment_header_bytes = int(segment_header_bytes)
        self.materialize = materialize
        self.read_only = read_only
        self.precreate_min_free_bytes = precreate_min_free_bytes
        self.store = None
        self._precreate_thread: threading.Thread | None = None
        self._stop = threading.Event()

    @property
    def fingerprint(self) -> bytes:
        return layout_fingerprint(self.namespace, self.segment_file_slots, self.segment_header_bytes)

    def open(self):
        if self.store is not None:
            return self.store
        if not self.read_only:
            self.root.mkdir(parents=True, exist_ok=True)
            for m in self.mounts:
                Path(m).mkdir(parents=True, exist_ok=True)
        s = core().ObjectStore()
        s.open({
            "uri": str(self.root),
            "segment_bytes": self.segment_bytes,
            "segment_count": self.segment_count,
            "segment_file_slots": self.segment_file_slots,
            "segment_header_bytes": self.segment_header_bytes,
            "capacity_slots": self.capacity_chunks,
            "fingerprint": self.fingerprint.decode("latin-1"),
            "mounts": self.mounts,
            "rank_id": self.rank,
            "rank_count": self.rank_count,
            "read_only": self.read_only,
            "materialize": self.materialize,
        })
        s.recover()
        self.store = s
        return s

    @staticmethod
    def open_view(root: str | os.PathLike, mounts: list[str] | None = None, rank: int = 0):
        """A read-only view of an existing namespace that takes its layout from the namespace itself.

        For a process that knows where the store lives but not the model (the vLLM
        scheduler at cold start): ``recover()`` lists the committed chunk keys,
        ``contains_prefix(keys, True)`` checks them on every rank's bitmap.
        """
        s = core().ObjectStore()
        mounts = [str(m) for m in (mounts or [root])]
        s.open({"uri": str(root), "segment_bytes": 4096, "segment_count": 1, "segment_file_slots": 1,
                "segment_header_bytes": 4096, "mounts": mounts, "rank_id": int(rank), "rank_count": int(rank) + 1,
                "read_only": True, "adopt_namespace_meta": True})
        return s

    def close(self) -> None:
        self.stop_background_precreate()
        if self.store is not None:
            self.store.close()
            self.store = None

    # -- growth -------------------------------------------------------------
    def _free_bytes(self) -> int:
        return min(shutil.disk_usage(m).free for m in self.mounts)

    def _min_free(self) -> int:
        if self.precreate_min_free_bytes is not None:
            return self.precreate_min_free_bytes
        total = min(shutil.disk_usage(m).total for m in self.mounts)
        return min(DEFAULT_PRECREATE_MIN_FREE_BYTES, total * 5 // 100)

    def precreate_until(self, slots: int) -> int:
        """Synchronously materialise file groups until ``slots`` are ready."""
        s = self.open()
        while s.ready_slots < min(slots, s.total_slots):
            if self._free_bytes() - s.file_bytes * len(self.mounts) < self._min_free():
                break
            if s.precreate_step(1 << 62) == 0:
                break
        return s.ready_slots

    def start_background_precreate(self, headroom: int | None = None, interval_s: float = 0.5) -> None:
        """Keep ``headroom`` free ready slots ahead of allocation (one file group at a time)."""
        s = self.open()
        group = self.segment_file_slots * len(self.mounts)
        headroom = group if headroom is None else headroom

        def run():
            while not self._stop.wait(interval_s):
                try:
                    if self._free_bytes() - s.file_bytes * len(self.mounts) < self._min_free():
                        continue
                    s.precreate_step(headroom)
                except Exception:  # pragma: no cover - logged by callers via usage()
                    continue

        self._stop.clear()
        self._precreate_thread = threading.Thread(target=run, name="tutti-precreate", daemon=True)
        self._precreate_thread.start()

    def stop_background_precreate(self) -> None:
        self._stop.set()
        if self._precreate_thread is not None:
            self._precreate_thread.join(timeout=10)
            self._precreate_thread = None
