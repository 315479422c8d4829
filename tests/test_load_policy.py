"""Load policy (sync / async / auto cost model) and the scheduler's load settlement."""
from types import SimpleNamespace

import pytest

from tutti_b200.integration.vllm.load_policy import LoadPolicy, resolve_free_ratio
from tutti_b200.integration.vllm.metadata import TuttiWorkerMetadata
from tutti_b200.integration.vllm.scheduler import SchedulerSide

BS, CHUNK = 4, 8
ROOMY = dict(held_blocks=0, need_blocks=10, free_blocks=1000)


def test_modes_and_gates():
    assert not LoadPolicy("sync").decide(chunks=100, compute_tokens=1, others=5, **ROOMY).is_async
    a = LoadPolicy("async")
    assert a.decide(chunks=1, compute_tokens=1, others=1, **ROOMY).is_async
    d = a.decide(chunks=1, compute_tokens=1, others=0, **ROOMY)
    assert not d.is_async and d.reason == "alone"
    d = a.decide(chunks=1, compute_tokens=1, others=3, held_blocks=400, need_blocks=200, free_blocks=500)
    assert not d.is_async and d.reason == "memory"  # 600 > 0.5 * (500 + 400)
    d = a.decide(chunks=1, compute_tokens=1, others=3, held_blocks=0, need_blocks=1, free_blocks=None)
    assert d.reason == "memory"  # unknown pool: stay synchronous
    assert a.decisions == {"async:mode=async": 1, "sync:alone": 1, "sync:memory": 2}
    with pytest.raises(ValueError):
        LoadPolicy("sometimes")


def test_auto_cost_rule_after_calibration():
    p = LoadPolicy("auto")
    assert p.decide(chunks=10, compute_tokens=100, others=4, **ROOMY).reason == "uncalibrated"
    p.observe_read(chunks=10, ms=50.0)  # 5 ms per chunk
    p.observe_step(tokens=100, ms=30.0)  # decode-sized: step time only
    assert p.compute_ms_per_token.value is None and p.step_ms.value == 30.0
    p.observe_step(tokens=1000, ms=40.0)  # prefill-sized: 0.04 ms per token
    assert p.compute_ms_per_token.value == pytest.approx(0.04)
    # long read (100 chunks = 500 ms) vs T = 0.04*1000 + S: sync would stall 4 others -> async
    d = p.decide(chunks=100, compute_tokens=1000, others=4, **ROOMY)
    assert d.is_async and d.reason == "cost" and d.read_ms == pytest.approx(500.0)
    # short read hides under the step -> sync
    assert not p.decide(chunks=2, compute_tokens=1000, others=4, **ROOMY).is_async


def test_free_ratio_resolution(monkeypatch):
    monkeypatch.delenv("TUTTI_ASYNC_LOAD_FREE_RATIO", raising=False)
    assert resolve_free_ratio({}) == 0.5 and resolve_free_ratio({"async_load_free_ratio": 0.25}) == 0.25
    monkeypatch.setenv("TUTTI_ASYNC_LOAD_FREE_RATIO", "0.75")
    assert resolve_free_ratio({"async_load_free_ratio": 0.25}) == 0.75
    monkeypatch.setenv("TUTTI_ASYNC_LOAD_FREE_RATIO", "2")
    with pytest.raises(ValueError):
        resolve_free_ratio({})


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
    assert s.policy.read_ms_per_chunk.value == pytest.approx(5.0)
    assert s.policy.step_ms.value == pytest.approx(45.0)
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
