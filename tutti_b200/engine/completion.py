"""Completion handles composed by the engine.

Parity: reference tutti/engine/completion.py:14-194 (aggregate and post
completions, LoadGateError carrying the failed chunk range).
"""
from __future__ import annotations

import time
from typing import Callable, Iterable


class LoadGateError(RuntimeError):
    """A restore failed; ``failed_chunks`` are indices into the plan's chunk list."""

    def __init__(self, message: str, failed_chunks: Iterable[int] = ()):
        super().__init__(message)
        self.failed_chunks = sorted(set(failed_chunks))


def settle_by(comp, deadline: float | None) -> bool:
    """Wait for ``comp`` until ``deadline`` (``time.monotonic()``; None: no limit).

    Returns False, without waiting further, when it is still running at the
    deadline; otherwise settles it (``wait``, which may raise its failure) and
    returns True. For shutdown paths that must not block on a stuck operation.
    """
    if deadline is not None:
        while not comp.query():
            if time.monotonic() >= deadline:
                return False
            time.sleep(0.001)
    comp.wait()
    return True


class AggregateCompletion:
    """Waits on several completions; the first error is raised after all were waited."""

    def __init__(self, parts: Iterable, on_done: Callable[[bool], None] | None = None):
        self._parts = list(parts)
        self._on_done = on_done
        self._done = False
        self.error: BaseException | None = None

    def query(self) -> bool:
        return self._done or all(p.query() for p in self._parts)

    def read_ms(self) -> float | None:
        """The slowest part's read time, once every part knows its own (entities read in parallel)."""
        times = [p.read_ms() if hasattr(p, "read_ms") else None for p in self._parts]
        return None if not times or any(t is None for t in times) else max(times)

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


class TimedCompletion:
    """A restore's completion and its read time.

    Device-timed between two events recorded on the IO stream around the
    submission (the io kernel runs until its data is in place). When the read
    finishes elsewhere (split completion: its drain is launched later, on
    another stream), the read time is the host time from submission to the
    first observation of completion instead. ``read_ms`` is None until known.
    """

    def __init__(self, inner, ev_start=None, ev_end=None, device_timed: bool = True, host_ms: float | None = None):
        self._inner = inner
        self._ev = (ev_start, ev_end) if device_timed and ev_start is not None else None
        self._t0 = time.perf_counter()
        self._host_ms: float | None = host_ms  # given when the read already finished (synchronous stores)

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def _mark(self) -> None:
        if self._host_ms is None:
            self._host_ms = (time.perf_counter() - self._t0) * 1e3

    def query(self) -> bool:
        done = self._inner.query()
        if done:
            self._mark()
        return done

    def wait(self, *a, **kw) -> None:
        try:
            self._inner.wait(*a, **kw)
        finally:
            self._mark()

    def enqueue_wait(self, stream=None) -> None:
        self._inner.enqueue_wait(stream)

    def read_ms(self) -> float | None:
        if self._ev is not None:
            start, end = self._ev
            return float(start.elapsed_time(end)) if end.query() else None
        return self._host_ms
