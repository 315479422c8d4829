"""Synchronous vs asynchronous load decision, from online measurements.

A synchronous load runs layerwise inside the request's first forward: layer
l's restore overlaps layer l-1's attention, and a read longer than the step
makes the whole batch (running decodes included) wait for the excess. An
asynchronous load parks the request in WAITING_FOR_REMOTE_KVS while the
other requests keep stepping; the request loses its own read/compute overlap
and holds its blocks idle for the whole read.

``decide`` (modes ``sync``, ``async``, ``auto``):

* ``sync``: always synchronous;
* ``async``: asynchronous when another request is computing and the blocks
  held by asynchronous loads (this one included) stay within ``free_ratio``
  of the blocks that computing requests do not use; otherwise synchronous;
* ``auto``: the same two gates, then a cost comparison. With ``R`` the
  estimated read time of this load, and ``T = C + S`` (``C``: this request's
  remaining compute, ``S``: the rest of a step)::

      synchronous cost  = max(0, R - T) * others   # every other request waits
      asynchronous cost = min(R, T)                # this request's lost overlap

  asynchronous iff the synchronous cost is larger. Until reads and prefill
  compute have been measured, loads stay synchronous.

``R``, ``C`` and ``S`` come from exponentially weighted averages of what the
workers measure: read ms per chunk (device-timed restores), compute ms per
token (steps of at least ``PREFILL_SAMPLE_TOKENS`` tokens without a
synchronous read) and step ms. The scheduler feeds the slowest rank's sample
of each step (TP ranks advance together).
Parity: reference tutti/integration/vllm/load_policy.py:1-180 (the same
modes, gates and cost rule; ``TUTTI_LOAD_MODE`` and
``TUTTI_ASYNC_LOAD_FREE_RATIO``).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

MODES = ("sync", "async", "auto")
DEFAULT_FREE_RATIO = 0.5
PREFILL_SAMPLE_TOKENS = 512  # shorter steps are decode-dominated: no prefill cost signal


def resolve_free_ratio(extra: dict | None = None) -> float:
    """``TUTTI_ASYNC_LOAD_FREE_RATIO`` > ``async_load_free_ratio`` in the connector config > 0.5."""
    raw = os.environ.get("TUTTI_ASYNC_LOAD_FREE_RATIO") or (extra or {}).get("async_load_free_ratio")
    if raw is None:
        return DEFAULT_FREE_RATIO
    ratio = float(raw)
    if not 0.0 < ratio <= 1.0:
        raise ValueError(f"async_load_free_ratio must be in (0, 1], got {raw!r}")
    return ratio


class Ewma:
    def __init__(self, alpha: float):
        self.alpha = alpha
        self.value: float | None = None

    def add(self, x: float) -> None:
        self.value = float(x) if self.value is None else self.value + self.alpha * (float(x) - self.value)


@dataclass
class LoadDecision:
    is_async: bool
    reason: str
    read_ms: float
    compute_ms: float
    step_ms: float


class LoadPolicy:
    def __init__(self, mode: str = "sync", free_ratio: float = DEFAULT_FREE_RATIO,
                 max_step_tokens: int | None = None, alpha: float = 0.2):
        if mode not in MODES:
            raise ValueError(f"load mode must be one of {MODES}, got {mode!r}")
        self.mode = mode
        self.free_ratio = float(free_ratio)
        self.max_step_tokens = int(max_step_tokens) if max_step_tokens else None
        self.read_ms_per_chunk = Ewma(alpha)
        self.compute_ms_per_token = Ewma(alpha)
        self.step_ms = Ewma(alpha)
        self.decisions: dict[str, int] = {}

    # -- measurements -----------------------------------------------------------
    def observe_read(self, chunks: int, ms: float) -> None:
        if chunks > 0 and ms > 0:
            self.read_ms_per_chunk.add(ms / chunks)

    def observe_step(self, tokens: int, ms: float) -> None:
        if tokens <= 0 or ms <= 0:
            return
        self.step_ms.add(ms)
        if tokens >= PREFILL_SAMPLE_TOKENS:
            self.compute_ms_per_token.add(ms / tokens)

    # -- decision ---------------------------------------------------------------
    def _memory_allows(self, held: int, need: int, free: int | None) -> bool:
        return free is not None and held + need <= self.free_ratio * (max(0, free) + held)

    def decide(self, *, chunks: int, compute_tokens: int, others: int, held_blocks: int, need_blocks: int,
               free_blocks: int | None) -> LoadDecision:
        """``others``: requests computing besides this one; ``held_blocks``: blocks held by asynchronous
        loads; ``need_blocks``: blocks this request holds once admitted; ``free_blocks``: estimated free
        blocks before admitting it (None: unknown, which keeps the load synchronous)."""
        tokens = max(0, int(compute_tokens))
        if self.max_step_tokens:
            tokens = min(tokens, self.max_step_tokens)
        r, c = self.read_ms_per_chunk.value, self.compute_ms_per_token.value
        step = self.step_ms.value or 0.0
        read_ms = r * chunks if r is not None else 0.0
        compute_ms = c * tokens if c is not None else 0.0
        if self.mode == "sync":
            is_async, reason = False, "mode=sync"
        elif others <= 0:
            is_async, reason = False, "alone"  # nobody computes while this request waits
        elif not self._memory_allows(held_blocks, need_blocks, free_blocks):
            is_async, reason = False, "memory"
        elif self.mode == "async":
            is_async, reason = True, "mode=async"
        elif r is None or c is None:
            is_async, reason = False, "uncalibrated"
        else:
            hidden = compute_ms + step
            is_async = max(0.0, read_ms - hidden) * others > min(read_ms, hidden)
            reason = "cost"
        key = ("async:" if is_async else "sync:") + reason
        self.decisions[key] = self.decisions.get(key, 0) + 1
        return LoadDecision(is_async, reason, read_ms, compute_ms, step)

    def snapshot(self) -> dict:
        return {"mode": self.mode, "free_ratio": self.free_ratio,
                "read_ms_per_chunk": self.read_ms_per_chunk.value,
                "compute_ms_per_token": self.compute_ms_per_token.value, "step_ms": self.step_ms.value,
                "decisions": dict(self.decisions)}
