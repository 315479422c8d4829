"""Load policy (sync / async / auto cost model) and the scheduler's load settlement."""
from types import SimpleNamespace

import pytest

from tutti_b200.integration.vllm.load_policy import LineFit, LoadPolicy, free_ratio_setting
from tutti_b200.integration.vllm.metadata import TuttiWorkerMetadata
from tutti_b200.integration.vllm.scheduler import SchedulerSide

BS, CHUNK = 4, 8
ROOMY = dict(held_blocks=0, need_blocks=10, free_blocks=1000)


def test_modes_and_gates():
    assert not LoadPolicy("sync").decide(chunks=100, compute_tokens=1, others=5, **ROOMY).asynchronous
    a = LoadPolicy("async")
    assert a.decide(chunks=1, compute_tokens=1, others=1, **ROOMY).asynchronous
    d = a.decide(chunks=1, compute_tokens=1, others=0, **ROOMY)
    assert not d.asynchronous and d.basis == "alone"
    d = a.decide(chunks=1, compute_tokens=1, others=3, held_blocks=400, need_blocks=200, free_blocks=500)
    assert not d.asynchronous and d.basis == "memory"  # 600 > 0.5 * (500 + 400)
    d = a.decide(chunks=1, compute_tokens=1, others=3, held_blocks=0, need_blocks=1, free_blocks=None)
    assert d.basis == "memory"  # unknown pool: stay synchronous
    assert a.snapshot()["decisions"] == {"async/mode": 1, "sync/alone": 1, "sync/memory": 2}
    with pytest.raises(ValueError):
        LoadPolicy("sometimes")


def test_line_fit_cases():
    f = LineFit()
    assert f.line() is None and f.at(3) is None
    f.add(10, 50.0)  # one x: proportional through the origin
    assert f.line() == (0.0, 5.0)
    g = LineFit(half_life=1e9)
    for x in (100, 1000, 400):
        g.add(x, 30.0 + x / 90.0)
    a, b = g.line()
    assert a == pytest.approx(30.0) and b == pytest.approx(1 / 90.0)
    h = LineFit(half_life=1e9)
    h.add(1, 10.0)
    h.add(5, 2.0)  # cost falling with size is not believed: the mean
    assert h.line() == pytest.approx((6.0, 0.0))
    k = LineFit(half_life=1.0)  # the newest sample weighs twice the one before
    k.add(1, 1.0)
    k.add(1, 4.0)
    assert k.at(1) == pytest.approx(3.0)


def test_auto_cost_rule_after_calibration():
    p = LoadPolicy("auto")
    assert p.decide(chunks=10, compute_tokens=100, others=4, **ROOMY).basis == "uncalibrated"
    p.record_restore(chunks=10, ms=50.0)  # 5 ms per chunk
    assert p.restore_ms(100) == pytest.approx(500.0)
    assert p.decide(chunks=10, compute_tokens=100, others=4, **ROOMY).basis == "uncalibrated"  # no steps yet
    p.record_step(tokens=100, ms=30.0)
    p.record_step(tokens=1000, ms=40.0)
    s0, s1 = p.steps.line()
    assert s1 > 0 and s0 + s1 * 1000 == pytest.approx(40.0, rel=0.05)
    # 100 chunks (500 ms) against a window of this request's 1000 tokens plus one typical step:
    # a synchronous read would stall 4 others far longer than waiting costs this request
    d = p.decide(chunks=100, compute_tokens=1000, others=4, **ROOMY)
    assert d.asynchronous and d.basis == "cost" and d.read_ms == pytest.approx(500.0)
    assert d.window_ms == pytest.approx(s1 * 1000 + p.step_ms(p.steps.mean_x))
    # a short read hides under the window -> synchronous
    assert not p.decide(chunks=2, compute_tokens=1000, others=4, **ROOMY).asynchronous


def test_free_ratio_setting(monkeypatch):
    monkeypatch.delenv("TUTTI_ASYNC_LOAD_FREE_RATIO", raising=False)
    assert free_ratio_setting({}) == 0.5 and free_ratio_setting({"async_load_free_ratio": 0.25}) == 0.25
    monkeypatch.setenv("TUTTI_ASYNC_LOAD_FREE_RATIO", "0.75")
    assert free_ratio_setting({"async_load_free_ratio": 0.25}) == 0.75
    monkeypatch.setenv("TUTTI_ASYNC_LOAD_FREE_RATIO", "2")
    with pytest.raises(ValueError):
        free_ratio_setting({})


def _resident_request(s, rid, n, base=0, status="RUNNING"):
    r = SimpleNamespace(request_id=rid, prompt_token_ids=list(range(base, base + n)), num_computed_tokens=0,
                        status=SimpleNamespace(name=status))
    s.get_num_new_matched_tokens(r, 0)
    keys = s.requests[rid].keys
    s.index.plan_store(keys)
    s.index.confirm_store(keys)
    return r, keys


def test_sync_load_settles_with_its_step_and_failed_chunks_are_forgotten():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64)
    r, keys = _resident_request(s, "a", 25)  # 3 chunks, 24 loadable
    ext, is_async = s.get_num_new_matched_tokens(r, 0)
    assert (ext, is_async) == (24, False)
    s.update_state_after_alloc(r, list(range(7)), ext)
    meta = s.build_meta([("a", list(range(7)), 0, 1)])
    assert meta.loads and meta.step_tokens == 1 and all(s.index.is_pinned(k) for k in keys)
    # the worker reports chunk 1 (token 8) failed in that step
    s.update_from_workers(TuttiWorkerMetadata(failed_loads={"a": 8}, generation=meta.generation))
    assert not any(s.index.is_pinned(k) for k in keys)
    assert s.index.is_resident(keys[0]) and not s.index.is_resident(keys[1]) and not s.index.is_resident(keys[2])
    assert s.profile["loads_failed"] == 1


def test_async_load_settles_when_received_and_counts_held_blocks():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64, total_blocks=100, policy=LoadPolicy("async"))
    other, _ = _resident_request(s, "busy", 9, base=5000)
    other.num_computed_tokens = 40  # 10 blocks in use
    s.update_state_after_alloc(other, [], 0)
    r, keys = _resident_request(s, "a", 17)
    ext, is_async = s.get_num_new_matched_tokens(r, 0)
    assert ext == 16 and is_async
    s.update_state_after_alloc(r, [1, 2, 3, 4, 5], ext, is_async=True)
    assert s._block_usage("x") == (1, 4, 100 - 10 - 4)
    meta = s.build_meta([])
    assert meta.loads[0].is_async
    s.update_from_workers(None, finished_recving={"a"})
    assert not any(s.index.is_pinned(k) for k in keys) and s._async_blocks == {}
    assert s.profile["loads_ok"] == 1


def test_policy_learns_from_the_slowest_rank():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64, policy=LoadPolicy("auto"))
    a = TuttiWorkerMetadata(read_samples=[(10, 20.0)], step_samples=[(600, 30.0)])
    b = TuttiWorkerMetadata(read_samples=[(10, 50.0)], step_samples=[(600, 45.0)])
    s.update_from_workers(a.aggregate(b))
    assert s.policy.restore_ms(1) == pytest.approx(5.0)  # the slower rank's 50 ms for 10 chunks
    assert s.policy.step_ms(600) == pytest.approx(45.0)
    assert s.maybe_log(force=True)


def test_stale_pending_saves_are_reclaimed_by_the_step_loop():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64)
    r = SimpleNamespace(request_id="a", prompt_token_ids=list(range(17)), num_computed_tokens=0)
    s.get_num_new_matched_tokens(r, 0)
    s.update_state_after_alloc(r, list(range(5)), 0)
    meta = s.build_meta([("a", list(range(5)), 0, 17)])
    k = meta.saves[0].keys
    assert all(s.index.is_pending(x) for x in k)
    for _ in range(70):  # no rank ever reports the save
        s.build_meta([])
    assert not any(s.index.is_pending(x) for x in k)


def test_retrieve_limits():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64, min_retrieve_tokens=17, max_tokens_per_load=20)
    r, _ = _resident_request(s, "a", 41)  # 5 chunks, 40 loadable
    assert s.get_num_new_matched_tokens(r, 0)[0] == 16  # capped at 20 -> whole chunks: 16
    assert s.get_num_new_matched_tokens(r, 24)[0] == 0  # the 16 tokens left are below the minimum
    s2 = SchedulerSide(BS, CHUNK, capacity_chunks=64, min_retrieve_tokens=17)
    r2, _ = _resident_request(s2, "b", 17)
    assert s2.get_num_new_matched_tokens(r2, 0)[0] == 0  # a 16-token hit is below the minimum
