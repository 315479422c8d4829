"""Completion handles composed by the engine.

Parity: reference tutti/engine/completion.py:14-194 (aggregate and post
completions, LoadGateError carrying the failed chunk range).
"""
from __future__ import annotations

from typing import Callable, Iterable


class LoadGateError(RuntimeError):
    """A restore failed; ``failed_chunks`` are indices into the plan's chunk list."""

    def __init__(self, message: str, failed_chunks: Iterable[int] = ()):
        super().__init__(message)
        self.failed_chunks = sorted(set(failed_chunks))


class AggregateCompletion:
    """Waits on several completions; the first error is raised after all were waited."""

    def __init__(self, parts: Iterable, on_done: Callable[[bool], None] | None = None):
        self._parts = list(parts)
        self._on_done = on_done
        self._done = False
        self.error: BaseException | None = None

    def query(self) -> bool:
        return self._done or all(p.query() for p in self._parts)

    def wait(self) -> None:
        if self._done:
            if self.error:
                raise self.error
            return
        for p in self._parts:
            try:
                p.wait()
            except BaseException as e:  # noqa: BLE001 - re-raised below
                if self.error is None:
                    self.error = e
        self._done = True
        if self._on_done:
            self._on_done(self.error is None)
        if self.error:
            raise self.error


class PostCompletion:
    """Runs ``after`` once the wrapped completion succeeded (e.g. commit, confirm)."""

    def __init__(self, inner, after: Callable[[], None] | None = None, on_error: Callable[[], None] | None = None):
        self._inner = inner
        self._after = after
        self._on_error = on_error
        self._done = False

    def query(self) -> bool:
        return self._done or self._inner.query()

    def wait(self) -> None:
        if self._done:
            return
        try:
            self._inner.wait()
        except BaseException:
            self._done = True
            if self._on_error:
                self._on_error()
            raise
        self._done = True
        if self._after:
            self._after()
