"""Property tests (hypothesis) of the stateful host pieces: chunk index, object store, load settlement."""
import tempfile
from pathlib import Path
from types import SimpleNamespace

from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st
from hypothesis.stateful import RuleBasedStateMachine, invariant, rule

from tutti_b200._native import core
from tutti_b200.index.chunk_index import ChunkIndex
from tutti_b200.integration.vllm.load_policy import LoadPolicy
from tutti_b200.integration.vllm.metadata import TuttiWorkerMetadata
from tutti_b200.integration.vllm.scheduler import SchedulerSide

KEYS = [bytes([i]) * 16 for i in range(12)]
key_sets = st.lists(st.sampled_from(KEYS), min_size=1, max_size=6, unique=True)


class IndexMachine(RuleBasedStateMachine):
    """ChunkIndex against a plain model: capacity is never exceeded and pinned chunks are never evicted."""

    CAP = 5

    def __init__(self):
        super().__init__()
        self.idx = ChunkIndex(self.CAP, 16)
        self.resident, self.pending, self.pins = set(), set(), {}

    @rule(keys=key_sets)
    def plan(self, keys):
        before = (set(self.resident), set(self.pending))
        p = self.idx.plan_store(keys)
        if p is None:
            assert (self.state_resident(), self.state_pending()) == before  # a refusal changes nothing
            return
        assert not (set(p.evicted_keys) & set(keys))
        assert all(self.pins.get(k, 0) == 0 for k in p.evicted_keys)
        self.resident -= set(p.evicted_keys)
        self.pending |= set(p.new_keys)

    @rule(ok=st.booleans(), data=st.data())
    def confirm(self, ok, data):
        if not self.pending:
            return
        keys = data.draw(st.lists(st.sampled_from(sorted(self.pending)), min_size=1, unique=True))
        self.idx.confirm_store(keys, ok)
        self.pending -= set(keys)
        if ok:
            self.resident |= set(keys)

    @rule(data=st.data())
    def pin(self, data):
        if not self.resident:
            return
        k = data.draw(st.sampled_from(sorted(self.resident)))
        self.idx.pin([k])
        self.pins[k] = self.pins.get(k, 0) + 1

    @rule(data=st.data())
    def unpin(self, data):
        held = sorted(k for k, n in self.pins.items() if n)
        if not held:
            return
        k = data.draw(st.sampled_from(held))
        self.idx.unpin([k])
        self.pins[k] -= 1

    @rule(keys=key_sets)
    def forget(self, keys):
        dropped = set(self.idx.forget(keys))
        assert all(self.pins.get(k, 0) == 0 for k in dropped)
        self.resident -= dropped

    def state_resident(self):
        return {k for k in KEYS if self.idx.is_resident(k)}

    def state_pending(self):
        return {k for k in KEYS if self.idx.is_pending(k)}

    @invariant()
    def matches_model(self):
        assert self.state_resident() == self.resident
        assert self.state_pending() == self.pending
        assert len(self.resident) + len(self.pending) <= self.CAP
        assert all(self.idx.is_pinned(k) == (n > 0) for k, n in self.pins.items())


TestIndexMachine = IndexMachine.TestCase
TestIndexMachine.settings = settings(max_examples=60, stateful_step_count=40, deadline=None)


@settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(ops=st.lists(st.tuples(st.sampled_from(["commit", "abort", "release"]), key_sets), min_size=1, max_size=12))
def test_object_store_recovers_exactly_the_committed_objects(ops):
    with tempfile.TemporaryDirectory() as d:
        root = Path(d)
        c = {"uri": str(root), "segment_bytes": 4096, "segment_count": 2, "segment_file_slots": 4,
             "segment_header_bytes": 8192, "capacity_slots": 16, "fingerprint": "prop",
             "mounts": [str(root / "d0"), str(root / "d1")]}
        s = core().ObjectStore()
        s.open(c)
        committed = set()
        for op, keys in ops:
            keys = [k + b"xx" for k in keys]  # 18-byte io keys
            if op == "release":
                s.release(keys)
                committed -= set(keys)
                continue
            fresh = [k for k in keys if k not in committed]
            if not fresh:
                continue
            acc, rej = s.reserve(fresh)
            got = [a[0] for a in acc]
            if op == "commit":
                s.commit(got)
                committed |= set(got)
            else:
                s.abort(got)
        s.close()
        s2 = core().ObjectStore()
        s2.open(c)
        assert set(s2.recover()) == committed
        s2.close()


@settings(max_examples=40, deadline=None)
@given(plan=st.lists(st.tuples(st.booleans(), st.booleans(), st.integers(0, 3)), min_size=1, max_size=8))
def test_every_settled_load_releases_its_pins(plan):
    """Random loads (sync or async, ok or failing at some chunk): once settled, no chunk stays pinned."""
    s = SchedulerSide(4, 8, capacity_chunks=256, total_blocks=10_000, policy=LoadPolicy("async"))
    busy = SimpleNamespace(request_id="busy", prompt_token_ids=list(range(9000, 9009)), num_computed_tokens=8,
                           status=SimpleNamespace(name="RUNNING"))
    s.update_state_after_alloc(busy, [], 0)
    received, failed = set(), {}
    for i, (want_async, ok, bad_chunk) in enumerate(plan):
        rid = f"r{i}"
        r = SimpleNamespace(request_id=rid, prompt_token_ids=list(range(i * 100, i * 100 + 33)),
                            num_computed_tokens=0, status=SimpleNamespace(name="WAITING"))
        s.get_num_new_matched_tokens(r, 0)
        keys = s.requests[rid].keys
        s.index.plan_store(keys)
        s.index.confirm_store(keys)
        ext, is_async = s.get_num_new_matched_tokens(r, 0)
        is_async = is_async and want_async
        s.update_state_after_alloc(r, list(range(i * 10, i * 10 + 9)), ext, is_async=is_async)
        if is_async:
            received.add(rid)
        if not ok:
            failed[rid] = bad_chunk * 8
    meta = s.build_meta([])
    s.update_from_workers(TuttiWorkerMetadata(failed_loads=failed, generation=meta.generation), received)
    assert s.index.stats()["pinned"] == 0
    for rid, first in failed.items():
        keys = s.requests[rid].keys
        assert all(not s.index.is_resident(k) for k in keys[first // 8:4])
