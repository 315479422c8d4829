"""vLLM connector: scheduler planning, worker load/save cycles, TP failure consensus (CPU)."""
import os
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tutti_b200.integration.vllm.metadata import LoadSpec, SaveSpec, TuttiConnectorMetadata, TuttiWorkerMetadata
from tutti_b200.integration.vllm.scheduler import SchedulerSide
from tutti_b200.integration.vllm.worker import WorkerSide
from tutti_b200.integration.vllm.factory import ConnectorConfig, make_engine, parse_bytes
from tutti_b200.parallel.tp_consensus import ChunkFailure, TpFailureConsensus, encode_row, merge_rows

BS, CHUNK = 4, 8  # 2 blocks per chunk


def req(rid, n, base=0):
    return SimpleNamespace(request_id=rid, prompt_token_ids=list(range(base, base + n)), num_computed_tokens=0)


def test_scheduler_match_alignment_and_one_token_rule():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64)
    r = req("a", 24)
    assert s.get_num_new_matched_tokens(r, 0) == (0, False)
    keys = s.requests["a"].keys
    assert len(keys) == 3
    s.index.plan_store(keys)
    s.index.confirm_store(keys)
    # 24 tokens fully resident: still leave one token to compute -> 16
    assert s.get_num_new_matched_tokens(r, 0) == (16, False)
    # already computed 8 -> 8 more
    assert s.get_num_new_matched_tokens(r, 8)[0] == 8
    # mid-chunk computed -> no load
    assert s.get_num_new_matched_tokens(r, 5)[0] == 0


def test_scheduler_saves_published_only_when_all_ranks_commit():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64, tp_size=2)
    r = req("a", 17)
    s.get_num_new_matched_tokens(r, 0)
    s.update_state_after_alloc(r, list(range(10, 15)), 0)
    meta = s.build_meta([("a", list(range(10, 15)), 0, 17)])
    assert len(meta.saves) == 1 and len(meta.saves[0].keys) == 2
    assert meta.saves[0].block_ids == [10, 11, 12, 13]
    k0, k1 = meta.saves[0].keys
    s.update_from_workers(TuttiWorkerMetadata({k0: 1, k1: 2}))
    assert not s.index.is_resident(k0) and s.index.is_resident(k1)
    s.update_from_workers(TuttiWorkerMetadata({k0: 1}).aggregate(TuttiWorkerMetadata({k0: 1})))
    assert s.index.is_resident(k0)
    # nothing new to save for the same request
    assert s.build_meta([("a", list(range(10, 15)), 17, 1)]).saves == []


def test_scheduler_load_spec_pins_until_finished():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=2)
    r = req("a", 17)
    s.get_num_new_matched_tokens(r, 0)
    keys = s.requests["a"].keys
    s.index.plan_store(keys)
    s.index.confirm_store(keys)
    ext, _ = s.get_num_new_matched_tokens(r, 0)
    s.update_state_after_alloc(r, [7, 8, 9, 10, 11], ext)
    meta = s.build_meta([])
    assert meta.loads[0].keys == keys and meta.loads[0].block_ids == [7, 8, 9, 10]
    assert s.index.is_pinned(keys[0])
    assert s.index.plan_store([b"x" * 16, b"y" * 16]) is None  # pinned keys are never evicted
    s.load_finished("a", keys, ok=True)
    assert not s.index.is_pinned(keys[0])


def make_worker(layers):
    cfg = ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "store": {"type": "memory", "capacity_chunks": 64}})
    w = WorkerSide(lambda t: make_engine(cfg, t, 0, 0, 1), block_size=BS, chunk_tokens=CHUNK)
    w.register_kv_caches({f"model.layers.{i}.self_attn.attn": t for i, t in enumerate(layers)})
    return w


def test_worker_save_then_load_roundtrip_cpu():
    layers = [torch.randn(2, 32, BS, 2, 16) for _ in range(3)]
    w = make_worker(layers)
    keys = [bytes([i]) * 16 for i in range(2)]
    wm = w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", keys, [0, 1, 2, 3])]))
    assert wm.committed == {keys[0]: 1, keys[1]: 1}
    ref = [t[:, 0:4].clone() for t in layers]
    meta = TuttiConnectorMetadata(2, [LoadSpec("b", keys, [20, 21, 22, 23], 16)], [])
    w.start_load_kv(meta)
    for i in range(3):
        w.wait_for_layer_load(f"model.layers.{i}.self_attn.attn")
    wm = w.wait_for_save(meta)
    for i in range(3):
        assert torch.equal(layers[i][:, 20:24], ref[i])
    assert w.get_block_ids_with_load_errors() == set()
    # the finished load is reported to the scheduler's load policy, with the step it ran in
    assert wm.generation == 2 and len(wm.read_samples) == 1 and wm.read_samples[0][0] == 2


def test_worker_reports_load_error_blocks():
    layers = [torch.randn(2, 32, BS, 2, 16) for _ in range(2)]
    w = make_worker(layers)
    missing = [b"m" * 16, b"n" * 16]
    meta = TuttiConnectorMetadata(5, [LoadSpec("r", missing, [8, 9, 10, 11], 16)], [])
    w.start_load_kv(meta)
    wm = w.wait_for_save(meta)
    assert wm.failed_loads == {"r": 0}
    assert w.get_block_ids_with_load_errors() == {8, 9, 10, 11}


def test_consensus_merge_rows():
    rows = [encode_row(7, 3, [ChunkFailure(1, 4, 2)]), encode_row(7, 3, [ChunkFailure(1, 2, 1), ChunkFailure(2, 0, 1)]),
            encode_row(7, 3, [])]
    c = merge_rows(7, 3, rows)
    assert c.failed and c.consistent
    assert list(c.failed_chunks(1)) == [2, 3, 4, 5] and list(c.failed_chunks(2)) == [0]
    assert not merge_rows(7, 3, [encode_row(7, 3, [])] * 2).failed
    assert merge_rows(7, 3, [encode_row(7, 3, []), encode_row(8, 3, [])]).failed  # generation skew


def _consensus_rank(rank, world, port, q, absent):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if rank == absent:
            q.put((rank, "absent"))
            return  # this rank never joins the collective
        c = TpFailureConsensus(timeout_s=3.0)
        try:
            failures = [ChunkFailure(0, 3, 2)] if rank == 1 else []
            res = c.coordinate(11, 2, failures)
            ok = c.drain_barrier(11, True) if res.failed else True
            q.put((rank, (res.failed, tuple(res.failed_chunks(0)), ok)))
        except Exception as e:  # noqa: BLE001
            q.put((rank, type(e).__name__))
    finally:
        pass


def _run(world, absent):
    import socket

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_consensus_rank, args=(r, world, port, q, absent)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=60) for _ in range(world))
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_consensus_two_gloo_ranks_agree():
    out = _run(2, absent=-1)
    assert out[0] == out[1] == (True, (3, 4), True)


def test_consensus_missing_rank_times_out():
    out = _run(2, absent=1)
    assert out[1] == "absent"
    assert out[0] in ("TimeoutError", "RuntimeError", "DistBackendError")


def test_config_parsing():
    c = ConnectorConfig.from_extra({"chunk_tokens": 512, "load_mode": "auto",
                                    "store": {"root": "/r/{LOCAL_RANK}", "capacity": "2GiB"}})
    assert c.chunk_tokens == 512 and c.capacity_bytes == 2 << 30
    assert parse_bytes("1.5 GB") == 1_500_000_000
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"bogus": 1})
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"store": {"type": "s3"}})
    c = ConnectorConfig.from_extra({"store": {"stored_format": "fp8_block128",
                                              "runtime_options": {"async_completion": True}}})
    assert c.stored_format == "fp8_block128" and c.runtime_options["async_completion"]
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"store": {"stored_format": "int4"}})


def test_connector_class_with_vllm_base():
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole

    from tutti_b200.integration.vllm.connector import TuttiConnectorV1

    cfg = SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_connector_extra_config={"chunk_tokens": CHUNK}),
                          cache_config=SimpleNamespace(block_size=BS),
                          parallel_config=SimpleNamespace(tensor_parallel_size=1))
    sch = TuttiConnectorV1(cfg, KVConnectorRole.SCHEDULER, None)
    r = req("q", 20)
    assert sch.get_num_new_matched_tokens(r, 0) == (0, False)
    out = SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(req_id="q", block_ids=([0, 1, 2, 3, 4],),
                                                              num_computed_tokens=0)],
                          num_scheduled_tokens={"q": 20}, scheduled_cached_reqs=None)
    meta = sch.build_connector_meta(out)
    assert len(meta.saves) == 1 and len(meta.saves[0].keys) == 2 and meta.step_tokens == 20
    # the step's output: both ranks' commits, no async receipts
    wm = TuttiWorkerMetadata({k: 1 for k in meta.saves[0].keys}, generation=meta.generation)
    sch.update_connector_output(SimpleNamespace(kv_connector_worker_meta=wm, finished_recving=None))
    assert all(sch._sched.index.is_resident(k) for k in meta.saves[0].keys)
    sch.update_connector_output(SimpleNamespace(kv_connector_worker_meta=None, finished_recving={"q"}))
    # vLLM's pool size reaches the load policy's block estimate
    sch2 = TuttiConnectorV1(cfg, KVConnectorRole.SCHEDULER, SimpleNamespace(num_blocks=1234))
    assert sch2._sched.total_blocks == 1234


def test_kv_layer_layouts_normalise_to_planes_first():
    from tutti_b200.integration.vllm.worker import normalize_kv_layer

    a = torch.zeros(2, 8, 16, 4, 64)
    na = normalize_kv_layer(a)
    assert na.shape == a.shape and na.data_ptr() == a.data_ptr() and na.is_contiguous()
    # heads-before-tokens inside each block (a permuted, still block-dense layout)
    raw = torch.arange(8 * 2 * 4 * 16 * 64, dtype=torch.float32).reshape(8, 2, 4, 16, 64)
    hnd = raw.permute(0, 1, 3, 2, 4)
    assert not hnd.is_contiguous()
    nh = normalize_kv_layer(hnd)
    assert nh.shape == (1, 8, 16, 8, 64) and torch.equal(nh[0, 5].reshape(-1), raw[5].reshape(-1))
    b = torch.arange(8 * 2 * 16 * 4 * 64, dtype=torch.float32).reshape(8, 2, 16, 4, 64)
    nb = normalize_kv_layer(b)
    assert nb.shape == (1, 8, 16, 8, 64) and nb.data_ptr() == b.data_ptr()
    # block 3's bytes (its K and V) are block 3 of the single plane
    assert torch.equal(nb[0, 3].reshape(-1), b[3].reshape(-1))
    m = normalize_kv_layer(torch.zeros(8, 64, 576))
    assert m.shape == (1, 8, 64, 1, 576)
    with pytest.raises(ValueError):  # blocks interleaved with planes: not one range per block
        normalize_kv_layer(torch.zeros(2, 8, 16, 4, 64).transpose(0, 1))


def test_reference_config_schema_and_import_path():
    import json as _json
    import os as _os

    ref_cfg = {"chunk_tokens": 512, "store": {"type": "tutti_nvme", "options": {
        "root": "/mnt/kv/tutti-kv-{LOCAL_RANK}", "capacity": "64 GiB",
        "preset": {"type": "raid0", "daemon_config": ["d.yaml"], "gpu_id": "{LOCAL_RANK}",
                   "device_groups": [[0, 1]]}}}}
    c = ConnectorConfig.from_extra(ref_cfg)
    assert c.store_type == "tutti" and c.root == "/mnt/kv/tutti-kv-{LOCAL_RANK}" and c.capacity_bytes == 64 << 30
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"store": {"type": "tutti_nvme", "options": {"bogus": 1}}})
    # vLLM resolves the connector class from the reference's module path
    import importlib

    mod = importlib.import_module("tutti.integration.vllm.connector")
    from tutti_b200.integration.vllm.connector import TuttiConnectorV1

    assert mod.TuttiConnectorV1 is TuttiConnectorV1


def test_worker_with_main_kv_and_index_cache_entities():
    # 3 attention layers, each with a main KV [2, nb, block, heads, dim] and an index cache [nb, block, 132] (uint8)
    cfg = ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "store": {"type": "memory", "capacity_chunks": 64}})
    w = WorkerSide(lambda t, entity="": make_engine(cfg, t, 0, 0, 1, entity), block_size=BS, chunk_tokens=CHUNK)
    main = [torch.randn(2, 32, BS, 2, 16) for _ in range(3)]
    index = [torch.randint(0, 256, (32, BS, 132), dtype=torch.uint8) for _ in range(3)]
    caches = {}
    for i in range(3):
        caches[f"model.layers.{i}.self_attn.attn"] = main[i]
        caches[f"model.layers.{i}.self_attn.indexer.k_cache"] = index[i]
    w.register_kv_caches(caches)
    assert w.engine.names == ["self_attn.attn", "self_attn.indexer.k_cache"] or len(w.engine.engines) == 2
    keys = [bytes([i + 40]) * 16 for i in range(2)]
    wm = w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", keys, [0, 1, 2, 3])]))
    assert wm.committed == {keys[0]: 1, keys[1]: 1}
    ref_m = [t[:, 0:4].clone() for t in main]
    ref_i = [t[0:4].clone() for t in index]
    meta = TuttiConnectorMetadata(2, [LoadSpec("b", keys, [20, 21, 22, 23], 16)], [])
    w.start_load_kv(meta)
    for name in caches:
        w.wait_for_layer_load(name)
    w.wait_for_save(meta)
    for i in range(3):
        assert torch.equal(main[i][:, 20:24], ref_m[i])
        assert torch.equal(index[i][20:24], ref_i[i])
    assert w.get_block_ids_with_load_errors() == set()


def test_lookahead_option():
    assert ConnectorConfig.from_extra({"lookahead_k": 2}).lookahead_k == 2
    assert ConnectorConfig.from_extra({}).lookahead_k == 4
    for bad in (0, -1, True, "3"):
        with pytest.raises(ValueError):
            ConnectorConfig.from_extra({"lookahead_k": bad})


def test_tutti_geometry_keys_are_checked():
    layers = [torch.zeros(2, 8, BS, 2, 16) for _ in range(3)]
    ok = ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "num_layers": 3, "physical_chunk_tokens": CHUNK,
                                     "max_chunks_per_wave": 64, "replica_io": True,
                                     "store": {"type": "memory", "capacity_chunks": 8}})
    make_engine(ok, layers, 0, 0, 1)
    bad = ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "num_layers": 4, "store": {"type": "memory"}})
    with pytest.raises(ValueError, match="num_layers"):
        make_engine(bad, layers, 0, 0, 1)
    direct = ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "direct_transfer": True, "store": {"type": "memory"}})
    with pytest.raises(ValueError, match="direct_transfer"):
        make_engine(direct, layers, 0, 0, 1)
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"chunk_tokens": CHUNK, "physical_chunk_tokens": 2 * CHUNK})
    with pytest.raises(ValueError):
        ConnectorConfig.from_extra({"store": {"type": "tutti_nvme", "options": {"segment_header_bytes": 100}}})
    assert ConnectorConfig.from_extra({"store": {"options": {"segment_header_bytes": 8192}}}).segment_header_bytes == 8192


class _SaveGate:
    """A save's completion whose device work finishes when the test says so."""

    def __init__(self):
        self.done = False
        self.waited_before_done = False

    def query(self):
        return self.done

    def wait(self):
        if not self.done:  # a real completion would block here until the write finished
            self.waited_before_done = True
            self.done = True


class _SaveEngine:
    staged = True  # no CUDA event on a CPU host

    def __init__(self):
        self.gates = []
        self.index = SimpleNamespace(is_resident=lambda k: False)
        self.store = SimpleNamespace()

    def store_chunks(self, keys, block_table, after=None):
        g = _SaveGate()
        self.gates.append(g)
        return g


def _saving_worker(max_inflight=64):
    w = WorkerSide(lambda t: None, block_size=BS, chunk_tokens=CHUNK, max_inflight_saves=max_inflight)
    w.engine = _SaveEngine()
    return w


def test_worker_step_does_not_wait_for_its_own_saves():
    w = _saving_worker()
    keys = [b"s" * 16, b"t" * 16]
    wm = w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", keys, [0, 1, 2, 3])]))
    gate = w.engine.gates[0]
    assert not gate.waited_before_done and wm.committed == {} and w.saves_in_flight() == 1
    # the request finished; the next step names it (its blocks may be reused) and goes on
    w.start_load_kv(TuttiConnectorMetadata(2, [], [], finished_saving=["a"]))
    assert w.get_finished({"a"}) == (None, None) and not gate.waited_before_done
    gate.done = True  # the write finished on the device
    wm = w.wait_for_save(TuttiConnectorMetadata(2, [], []))
    assert wm.committed == {keys[0]: 1, keys[1]: 1} and w.saves_in_flight() == 0


def test_worker_saves_settle_from_get_finished_and_in_any_order():
    w = _saving_worker()
    w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", [b"a" * 16], [0, 1]),
                                                   SaveSpec("b", [b"b" * 16], [2, 3])]))
    ga, gb = w.engine.gates
    gb.done = True
    w.get_finished({"a", "b"})  # b settles here, a stays in flight
    assert w.saves_in_flight() == 1
    ga.done = True
    wm = w.wait_for_save(TuttiConnectorMetadata(2, [], []))
    assert w.saves_in_flight() == 0 and set(wm.committed) == {b"a" * 16, b"b" * 16}
    assert not ga.waited_before_done and not gb.waited_before_done


def test_worker_back_pressure_waits_for_the_oldest_save_only():
    w = _saving_worker(max_inflight=2)
    for i in range(3):
        w.wait_for_save(TuttiConnectorMetadata(i + 1, [], [SaveSpec(f"r{i}", [bytes([i]) * 16], [0, 1])]))
    g0, g1, g2 = w.engine.gates
    assert g0.waited_before_done and not g1.waited_before_done and not g2.waited_before_done
    assert w.saves_in_flight() == 2
    w.engine.wait_idle = lambda timeout_s=None: None
    w.engine.store = SimpleNamespace()
    g1.done = g2.done = True  # their writes finished on the device
    w.shutdown()  # settles (commits) everything still in flight
    assert w.saves_in_flight() == 0 and g2.done


def test_worker_settle_saves_commits_every_save_in_flight():
    w = _saving_worker()
    w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", [b"a" * 16], [0, 1]),
                                                   SaveSpec("b", [b"b" * 16], [2, 3])]))
    assert w.saves_in_flight() == 2
    assert w.settle_saves() == 2 and w.saves_in_flight() == 0
    assert all(g.done for g in w.engine.gates)
    # reported committed in the next step's metadata
    wm = w.wait_for_save(TuttiConnectorMetadata(2, [], []))
    assert set(wm.committed) == {b"a" * 16, b"b" * 16}


def test_scheduler_names_finished_requests_whose_saves_may_be_in_flight():
    s = SchedulerSide(BS, CHUNK, capacity_chunks=64)
    for rid in ("a", "b"):
        r = req(rid, 17 if rid == "a" else 5, base=100 if rid == "b" else 0)
        s.get_num_new_matched_tokens(r, 0)
        s.update_state_after_alloc(r, list(range(10, 15)), 0)
    meta = s.build_meta([("a", list(range(10, 15)), 0, 17), ("b", list(range(20, 22)), 0, 5)])
    assert [sp.request_id for sp in meta.saves] == ["a"]  # b has no full chunk
    assert s.request_finished("a") is False and s.request_finished("b") is False  # blocks freed at once
    nxt = s.build_meta([])
    assert nxt.finished_saving == ["a"]  # the workers order this step's forward after a's saves
    assert s.build_meta([]).finished_saving == []


def test_worker_shutdown_does_not_wait_past_its_deadline_for_a_stuck_save():
    class _Stuck(_SaveGate):
        def wait(self):  # a save that never finishes would block here
            raise AssertionError("waited on a running save")

    w = _saving_worker()
    w.engine.store_chunks = lambda keys, bt, after=None: _Stuck()
    w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", [b"a" * 16], [0, 1])]))
    idle = []
    w.engine.wait_idle = lambda timeout_s=None: idle.append(timeout_s)
    t0 = __import__("time").monotonic()
    w.shutdown(timeout_s=0.2)
    assert __import__("time").monotonic() - t0 < 5.0
    assert w.saves_in_flight() == 1  # left uncommitted, not waited for
    assert idle and idle[0] <= 0.2


def test_worker_connector_passes_replica_options_from_the_model():
    """The worker role hands replica_io, its save mode and the model's KV-head count / MLA to the worker."""
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole

    from tutti_b200.integration.vllm.connector import TuttiConnectorV1

    extra = {"chunk_tokens": CHUNK, "replica_io": True, "replica_io_saves": "fanin"}
    mc = SimpleNamespace(use_mla=True, get_total_num_kv_heads=lambda: 1)
    cfg = SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_connector_extra_config=extra),
                          cache_config=SimpleNamespace(block_size=BS), model_config=mc,
                          parallel_config=SimpleNamespace(tensor_parallel_size=1))
    w = TuttiConnectorV1(cfg, KVConnectorRole.WORKER, None)._worker
    assert w.replica_io_saves == "fanin" and w.replica_kind == "latent" and w.kv_heads == 1
    assert w.replica_io is False  # TP 1: nothing to fan out
    cfg.kv_transfer_config.kv_connector_extra_config = dict(extra, replica_io_saves="nope")
    with pytest.raises(ValueError, match="replica_io_saves"):
        TuttiConnectorV1(cfg, KVConnectorRole.WORKER, None)
