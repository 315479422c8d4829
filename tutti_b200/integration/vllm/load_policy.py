"""When a prefix restore should hold its request back instead of running inline.

Two ways to load a request's cached prefix:

* synchronous: the restore runs inside the request's first forward, layer by
  layer (layer l's read overlaps layer l-1's attention). A read longer than
  the compute it hides under stalls the whole step, so every other request in
  the batch waits for the excess;
* asynchronous: the request waits (vLLM's WAITING_FOR_REMOTE_KVS) while the
  others keep stepping. It gives up the overlap with its own compute and holds
  its blocks idle for the whole read.

Cost model. Two straight lines are fitted online to what the workers measure,
each by weighted least squares with exponential forgetting (a sample's weight
halves every ``half_life`` samples, so the fit follows drifting load):

    restore_ms(chunks) = r0 + r1 * chunks     (device-timed restores)
    step_ms(tokens)    = s0 + s1 * tokens     (device-timed forward steps)

``r0``/``s0`` capture per-operation and per-step fixed costs (launches,
decode of the running batch), ``r1``/``s1`` the marginal costs. Decode-sized
steps are ordinary samples here: they pin down ``s0``. For a load of ``n``
chunks whose request still has ``m`` tokens to prefill, the read time is
``R = restore_ms(n)`` and the window that hides a synchronous read is
``W = s1 * m + step_ms(mean tokens of recent steps)`` (the request's own
prefill plus one typical step). Then::

    stall if synchronous   = max(0, R - W) * others
    loss if asynchronous   = min(R, W)

and the load goes asynchronous iff the stall exceeds the loss.

Modes: ``sync`` (always synchronous), ``async`` (asynchronous whenever the
gates allow) and ``auto`` (the gates, then the cost model; synchronous until
both fits have samples). Gates, in order: nobody else is computing (waiting
helps nobody), and the blocks held by asynchronous loads, this one included,
must stay within ``free_ratio`` of the blocks that computing requests leave.

Parity: the reference's policy (tutti/integration/vllm/load_policy.py) has the
same modes, the same two gates and the same stall-versus-loss comparison,
read from ``TUTTI_LOAD_MODE`` and ``TUTTI_ASYNC_LOAD_FREE_RATIO``; its
estimators are moving averages with a prefill-size cut-off, not fitted lines.
"""
from __future__ import annotations

import os
from collections import Counter
from typing import NamedTuple

MODES = ("sync", "async", "auto")
DEFAULT_FREE_RATIO = 0.5


def free_ratio_setting(extra: dict | None = None) -> float:
    """Share of free blocks asynchronous loads may hold.

    Precedence: the ``TUTTI_ASYNC_LOAD_FREE_RATIO`` environment variable, then
    ``async_load_free_ratio`` in the connector's extra config, then 0.5.
    """
    env = os.environ.get("TUTTI_ASYNC_LOAD_FREE_RATIO")
    raw = env if env else (extra or {}).get("async_load_free_ratio")
    if raw is None:
        return DEFAULT_FREE_RATIO
    value = float(raw)
    if value <= 0.0 or value > 1.0:
        raise ValueError(f"async_load_free_ratio must be in (0, 1], got {raw!r}")
    return value


class LineFit:
    """Online fit of ``y = a + b * x`` with exponentially decaying sample weights.

    Keeps weighted sums (w, Σx, Σy, Σxx, Σxy). Degenerate cases: samples at a
    single x fit a line through the origin (cost proportional to size); a fit
    whose slope comes out negative is replaced by the mean (size does not make
    work cheaper); one whose intercept comes out negative is refitted through
    the origin.
    """

    def __init__(self, half_life: float = 32.0):
        if half_life <= 0:
            raise ValueError("half_life must be positive")
        self._keep = 0.5 ** (1.0 / half_life)
        self._w = self._x = self._y = self._xx = self._xy = 0.0

    def add(self, x: float, y: float) -> None:
        k = self._keep
        x, y = float(x), float(y)
        self._w = self._w * k + 1.0
        self._x = self._x * k + x
        self._y = self._y * k + y
        self._xx = self._xx * k + x * x
        self._xy = self._xy * k + x * y

    @property
    def weight(self) -> float:
        return self._w

    @property
    def mean_x(self) -> float | None:
        return self._x / self._w if self._w else None

    def line(self) -> tuple[float, float] | None:
        """(intercept, slope), or None before the first sample."""
        if not self._w:
            return None
        mx, my = self._x / self._w, self._y / self._w
        var = self._xx / self._w - mx * mx
        if var <= 1e-12 * max(1.0, mx * mx):
            return (0.0, my / mx) if mx > 0 else (my, 0.0)
        slope = (self._xy / self._w - mx * my) / var
        if slope < 0:
            return my, 0.0
        intercept = my - slope * mx
        if intercept < 0:
            return 0.0, (self._xy / self._xx if self._xx > 0 else 0.0)
        return intercept, slope

    def at(self, x: float) -> float | None:
        ab = self.line()
        return None if ab is None else ab[0] + ab[1] * float(x)


class LoadChoice(NamedTuple):
    asynchronous: bool
    basis: str          # which rule decided: mode, alone, memory, uncalibrated, cost
    read_ms: float      # estimated restore time of this load (0 before calibration)
    window_ms: float    # compute a synchronous read hides under (0 before calibration)


class LoadPolicy:
    def __init__(self, mode: str = "sync", free_ratio: float = DEFAULT_FREE_RATIO,
                 max_step_tokens: int | None = None, half_life: float = 32.0):
        if mode not in MODES:
            raise ValueError(f"load mode must be one of {MODES}, got {mode!r}")
        self.mode = mode
        self.free_ratio = float(free_ratio)
        self.max_step_tokens = int(max_step_tokens) if max_step_tokens else None
        self.restores = LineFit(half_life)  # ms vs chunks
        self.steps = LineFit(half_life)     # ms vs tokens
        self.tally: Counter[tuple[str, bool]] = Counter()

    # -- measurements ------------------------------------------------------------
    def record_restore(self, chunks: int, ms: float) -> None:
        """A device-timed restore of ``chunks`` chunks."""
        if chunks > 0 and ms > 0:
            self.restores.add(chunks, ms)

    def record_step(self, tokens: int, ms: float) -> None:
        """A device-timed forward step that computed ``tokens`` tokens."""
        if tokens > 0 and ms > 0:
            self.steps.add(tokens, ms)

    def restore_ms(self, chunks: int) -> float | None:
        return self.restores.at(chunks)

    def step_ms(self, tokens: int) -> float | None:
        return self.steps.at(tokens)

    # -- decision ------------------------------------------------------------------
    def _room_for(self, held: int, need: int, free: int | None) -> bool:
        if free is None:
            return False  # unknown pool: do not park blocks
        return held + need <= self.free_ratio * (max(0, free) + held)

    def _window_ms(self, tokens: int) -> float | None:
        line, typical = self.steps.line(), self.steps.mean_x
        if line is None or typical is None:
            return None
        return line[1] * tokens + line[0] + line[1] * typical

    def decide(self, *, chunks: int, compute_tokens: int, others: int, held_blocks: int, need_blocks: int,
               free_blocks: int | None) -> LoadChoice:
        """Choose the load mode of one request.

        ``others``: requests computing besides this one; ``held_blocks``: blocks
        held by asynchronous loads in flight; ``need_blocks``: blocks this
        request holds once admitted; ``free_blocks``: free blocks before it is
        admitted (None when unknown).
        """
        tokens = max(0, int(compute_tokens))
        if self.max_step_tokens:
            tokens = min(tokens, self.max_step_tokens)
        read = self.restore_ms(chunks)
        window = self._window_ms(tokens)
        estimate = (read or 0.0, window or 0.0)
        if self.mode == "sync":
            choice = LoadChoice(False, "mode", *estimate)
        elif others <= 0:
            choice = LoadChoice(False, "alone", *estimate)
        elif not self._room_for(held_blocks, need_blocks, free_blocks):
            choice = LoadChoice(False, "memory", *estimate)
        elif self.mode == "async":
            choice = LoadChoice(True, "mode", *estimate)
        elif read is None or window is None:
            choice = LoadChoice(False, "uncalibrated", *estimate)
        else:
            stall = max(0.0, read - window) * others
            loss = min(read, window)
            choice = LoadChoice(stall > loss, "cost", read, window)
        self.tally[(choice.basis, choice.asynchronous)] += 1
        return choice

    def snapshot(self) -> dict:
        r, s = self.restores.line(), self.steps.line()
        return {
            "mode": self.mode, "free_ratio": self.free_ratio,
            "restore_ms": None if r is None else f"{r[0]:.3f}+{r[1]:.4f}/chunk",
            "step_ms": None if s is None else f"{s[0]:.3f}+{s[1]:.5f}/token",
            "decisions": {f"{'async' if a else 'sync'}/{b}": n for (b, a), n in sorted(self.tally.items())},
        }
