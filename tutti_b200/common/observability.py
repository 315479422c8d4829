"""Tracing, metrics and health logs.

* NVTX ranges, opt-in with ``TUTTI_NVTX=1``: ``nvtx_range("tutti.restore|layers=32")``
  around requests, layer loads, transfers and completions (the native data path
  adds ``tutti.nvme_gpu.submit|op=...`` ranges under the same switch).
* Counters for bytes moved, operations and failures, exported through
  ``prometheus_client`` when ``TUTTI_METRICS_PORT`` is set (and always readable
  with ``metrics()``).
* A health line on the ``tutti_b200`` logger at most every
  ``TUTTI_HEALTH_INTERVAL_S`` seconds (default 30): in-flight operations, store
  usage, controller commands/bytes/errors and the bandwidth since the last line.
Parity: reference tutti/common/nvtx.py:25-77 (opt-in ranges) and
tutti/integration/vllm/connector.py:555-677 (health and profile logs).
"""
from __future__ import annotations

import collections
import contextlib
import logging
import os
import threading
import time

LOG = logging.getLogger("tutti_b200")

_NVTX = os.environ.get("TUTTI_NVTX", "0") not in ("", "0", "false", "False")


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def nvtx_range(name: str):
    """An NVTX range when ``TUTTI_NVTX=1``; free otherwise."""
    if not _NVTX:
        yield
        return
    import torch

    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class Metrics:
    """Process-wide counters (thread safe); mirrored to Prometheus when enabled."""

    NAMES = ("restore_bytes", "store_bytes", "restore_ops", "store_ops", "failed_ops", "failed_requests",
             "submit_retries")

    def __init__(self):
        self._mu = threading.Lock()
        self._v = {n: 0 for n in self.NAMES}
        self._windows: dict[str, collections.deque] = {}
        self._prom = None
        port = os.environ.get("TUTTI_METRICS_PORT")
        if port:
            try:
                import prometheus_client as pc

                self._prom = {n: pc.Counter(f"tutti_{n}_total", f"tutti_b200 {n.replace('_', ' ')}")
                              for n in self.NAMES}
                pc.start_http_server(int(port))
            except Exception as e:  # noqa: BLE001  (metrics must never break IO)
                LOG.warning("[tutti] metrics export disabled: %s", e)
                self._prom = None

    def add(self, name: str, value: int = 1) -> None:
        with self._mu:
            self._v[name] += int(value)
        if self._prom is not None:
            self._prom[name].inc(value)

    def snapshot(self) -> dict:
        with self._mu:
            return dict(self._v)

    # -- latency windows (the last WINDOW samples of each kind) -------------------
    WINDOW = 2048

    def observe(self, name: str, value_ms: float) -> None:
        with self._mu:
            w = self._windows.get(name)
            if w is None:
                w = self._windows[name] = collections.deque(maxlen=self.WINDOW)
            w.append(float(value_ms))

    def percentiles(self, name: str, qs=(0.5, 0.99)) -> dict[str, float] | None:
        """``{"p50": ..., "p99": ...}`` over the window (nearest rank), or None without samples."""
        with self._mu:
            w = sorted(self._windows.get(name, ()))
        if not w:
            return None
        return {f"p{round(q * 100)}": w[min(len(w) - 1, int(q * len(w)))] for q in qs}


_metrics: Metrics | None = None
_metrics_mu = threading.Lock()


def metrics() -> Metrics:
    global _metrics
    with _metrics_mu:
        if _metrics is None:
            _metrics = Metrics()
        return _metrics


def health_interval_s() -> float:
    """``TUTTI_HEALTH_INTERVAL_S`` (default 30, at least 1: the health lines must not flood the log)."""
    return max(1.0, float(os.environ.get("TUTTI_HEALTH_INTERVAL_S", "30") or 30))


class HealthReporter:
    """Logs one ``[tutti] health`` line at most every ``interval_s`` seconds when ``maybe_log`` is called."""

    def __init__(self, store=None, interval_s: float | None = None, clock=time.monotonic):
        self.store = store
        self.interval_s = health_interval_s() if interval_s is None else interval_s
        self._clock = clock
        self._last_t = clock()
        self._last = metrics().snapshot()

    def report(self) -> dict:
        now = self._clock()
        cur = metrics().snapshot()
        dt = max(now - self._last_t, 1e-9)
        out = {"restore_GBps": (cur["restore_bytes"] - self._last["restore_bytes"]) / dt / 1e9,
               "store_GBps": (cur["store_bytes"] - self._last["store_bytes"]) / dt / 1e9,
               "failed_ops": cur["failed_ops"], "ops": cur["restore_ops"] + cur["store_ops"]}
        for kind in ("restore", "store"):
            pct = metrics().percentiles(f"{kind}_ms")
            if pct:  # submit to first observed completion, per op
                out.update({f"{kind}_ms_{k}": v for k, v in pct.items()})
        st = self.store
        if st is not None:
            out["inflight"] = len(getattr(st, "_inflight", ()))
            objects = getattr(st, "objects", None)
            if objects is not None and hasattr(objects, "usage"):
                u = objects.usage()
                out["committed_GB"] = u["committed_bytes"] / 1e9
                out["capacity_GB"] = u["capacity_bytes"] / 1e9
            rt = getattr(st, "runtime", None)
            if rt is not None and hasattr(rt, "controller_stats"):
                cs = rt.controller_stats()
                out["controller_commands"] = sum(c["commands"] for c in cs)
                out["controller_errors"] = sum(c["errors"] for c in cs)
        self._last_t, self._last = now, cur
        return out

    def maybe_log(self, force: bool = False) -> dict | None:
        if not force and self._clock() - self._last_t < self.interval_s:
            return None
        r = self.report()
        LOG.info("[tutti] health " + " ".join(f"{k}={v:.3f}" if isinstance(v, float) else f"{k}={v}"
                                               for k, v in r.items()))
        return r
