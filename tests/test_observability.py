"""Metrics counters, health lines and the NVTX switch (host only)."""
import logging

from tutti_b200.common import observability as obs
from tutti_b200.storage.tutti_store import NativeCompletion


class _Rt:
    def __init__(self, ok=True):
        self.ok = ok

    def wait(self, io, timeout_ms):
        return {"ok": self.ok, "failed_request_indices": [] if self.ok else [0, 3], "failure_kind": "cq_timeout"}

    def release_io(self, io):
        pass


def test_completion_counts_bytes_and_failures():
    m = obs.metrics()
    before = m.snapshot()
    NativeCompletion(_Rt(), [1], nbytes=4096).wait()
    NativeCompletion(_Rt(), [2], nbytes=100, kind="store").wait()
    try:
        NativeCompletion(_Rt(ok=False), [3], nbytes=7).wait()
    except Exception:
        pass
    after = m.snapshot()
    assert after["restore_bytes"] - before["restore_bytes"] == 4096
    assert after["store_bytes"] - before["store_bytes"] == 100
    assert after["restore_ops"] - before["restore_ops"] == 2
    assert after["failed_ops"] - before["failed_ops"] == 1
    assert after["failed_requests"] - before["failed_requests"] == 2


def test_health_line_rate_limited_and_reports_bandwidth(caplog):
    t = [100.0]
    h = obs.HealthReporter(store=None, interval_s=30, clock=lambda: t[0])
    assert h.maybe_log() is None
    obs.metrics().add("restore_bytes", 3 * 10**9)
    t[0] += 30.0
    with caplog.at_level(logging.INFO, logger="tutti_b200"):
        r = h.maybe_log()
    assert r is not None and abs(r["restore_GBps"] - 0.1) < 1e-9
    assert any("[tutti] health" in rec.message for rec in caplog.records)


def test_nvtx_range_is_free_when_disabled():
    assert not obs.nvtx_enabled()
    with obs.nvtx_range("x"):
        pass


def test_environment_switches(monkeypatch):
    from tutti_b200.common.env import runtime_option_defaults
    from tutti_b200.integration.vllm.factory import ConnectorConfig

    monkeypatch.setenv("TUTTI_IO_TIMING", "1")
    monkeypatch.setenv("TUTTI_POOL_WORKERS", "48")
    assert runtime_option_defaults() == {"timing": True, "max_ctas_per_op": 48}
    monkeypatch.setenv("TUTTI_LOAD_MODE", "auto")
    assert ConnectorConfig.from_extra({}).load_mode == "auto"
    assert ConnectorConfig.from_extra({"load_mode": "sync"}).load_mode == "auto"  # the variable wins
    monkeypatch.delenv("TUTTI_LOAD_MODE")
    assert ConnectorConfig.from_extra({"load_mode": "async"}).load_mode == "async"
    assert ConnectorConfig.from_extra({}).load_mode == "sync"
    monkeypatch.delenv("TUTTI_IO_TIMING")
    monkeypatch.delenv("TUTTI_POOL_WORKERS")
    assert runtime_option_defaults() == {}


def test_write_ordering_and_prp_mode_switches(monkeypatch):
    import pytest

    from tutti_b200.common.env import prp_mode
    from tutti_b200.engine.core import resolve_defer_writes
    from tutti_b200.integration.vllm.factory import ConnectorConfig

    monkeypatch.delenv("TUTTI_DEFER_WRITES_AFTER_READS", raising=False)
    assert resolve_defer_writes(None) is True
    monkeypatch.setenv("TUTTI_DEFER_WRITES_AFTER_READS", "0")
    assert resolve_defer_writes(None) is False
    assert resolve_defer_writes(True) is True  # an explicit option wins over the variable
    with pytest.raises(ValueError):
        resolve_defer_writes("yes")
    cfg = ConnectorConfig.from_extra({"store": {"type": "tutti_nvme", "options": {"defer_writes_after_reads": False}}})
    assert cfg.defer_writes_after_reads is False
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"store": {"options": {"defer_writes_after_reads": 1}}})

    monkeypatch.delenv("TUTTI_PRP_MODE", raising=False)
    assert prp_mode() == "dynamic"
    monkeypatch.setenv("TUTTI_PRP_MODE", "FULL_PREBUILD")
    assert prp_mode() == "full_prebuild"
    monkeypatch.setenv("TUTTI_PRP_MODE", "lazy")
    with pytest.raises(ValueError):
        prp_mode()


def test_latency_percentiles_in_the_health_line():
    import tutti_b200.common.observability as obs

    fresh = obs.Metrics()
    for v in range(1, 101):
        fresh.observe("restore_ms", float(v))
    assert fresh.percentiles("restore_ms") == {"p50": 51.0, "p99": 100.0}
    assert fresh.percentiles("nothing_ms") is None
    m = obs.metrics()  # the process-wide one the health line reads
    m._windows.pop("restore_ms", None)
    for v in range(1, 101):
        m.observe("restore_ms", float(v))
    r = obs.HealthReporter(interval_s=0).report()
    assert r["restore_ms_p50"] == 51.0 and r["restore_ms_p99"] == 100.0


def test_health_interval_has_a_floor(monkeypatch):
    from tutti_b200.common.observability import health_interval_s

    monkeypatch.setenv("TUTTI_HEALTH_INTERVAL_S", "0")
    assert health_interval_s() == 1.0
    monkeypatch.setenv("TUTTI_HEALTH_INTERVAL_S", "12.5")
    assert health_interval_s() == 12.5
    monkeypatch.delenv("TUTTI_HEALTH_INTERVAL_S")
    assert health_interval_s() == 30.0
