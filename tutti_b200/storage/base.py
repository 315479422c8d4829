"""KVStore SPI: the contract between the KV engine and a persistence backend.

A batch is a list of ``(key, buffer_id, offset)`` entries; one call is one
batch and one underlying submission. ``register_buffer`` registers memory
(a staging ring or a whole paged pool) and returns a buffer id, or ``None``
when the backend cannot use that granularity (the engine then stages).
Parity: reference tutti/storage/base.py:15-56.
"""
from __future__ import annotations

from collections.abc import Iterable, Sequence
from typing import Protocol


class Completion(Protocol):
    def wait(self) -> None: ...

    def query(self) -> bool: ...


class KVStore(Protocol):
    @property
    def capacity_chunks(self) -> int: ...

    def open(self) -> None: ...

    def close(self) -> None: ...

    def register_buffer(self, buffer, granularity: int) -> int | None: ...

    # optional: drop a registration (engines reuse and replace their staging buffers)
    def unregister_buffer(self, buffer_id: int) -> None: ...

    def put_batch(self, batch: Sequence[tuple[bytes, int, int]]) -> Completion: ...

    def get_batch(self, batch: Sequence[tuple[bytes, int, int]]) -> Completion: ...

    def drop(self, keys: Sequence[bytes]) -> None: ...

    def scan(self) -> Iterable[bytes]: ...


class DoneCompletion:
    """A completion that is already terminal (synchronous backends)."""

    def __init__(self, error: BaseException | None = None):
        self._error = error

    def wait(self) -> None:
        if self._error is not None:
            raise self._error

    def query(self) -> bool:
        return True


class StoreIOError(RuntimeError):
    """A batch finished with failed requests; ``failed`` lists batch indices."""

    def __init__(self, message: str, failed: Sequence[int] = (), kind: str = "unknown"):
        super().__init__(message)
        self.failed = list(failed)
        self.kind = kind
