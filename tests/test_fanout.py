"""Drive-affine fan-out restore: placement exchange and share selection (gloo, CPU)
and the fused NVLink fan-out on two GPUs (local vs fan-out pools byte-equal)."""
import datetime
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tutti_b200.parallel.fanout import FanoutRestorer, RestoreItem, owner_of

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_owner_of_is_le64_prefix_mod_group():
    k = bytes(range(16))
    assert owner_of(k, 8) == int.from_bytes(k[:8], "little") % 8
    assert owner_of(b"\x05" + b"\0" * 15, 4) == 1


class _Objects:
    def __init__(self, table, rank=0):
        self.table = table
        self.rank = rank
        self.reserved, self.committed, self.aborted = [], [], []

    def lookup(self, key):
        return self.table.get(key)

    def contains(self, key):
        return key in self.committed

    def reserve(self, keys):
        out = []
        for k in keys:
            i = k[0]
            out.append((k, f"file:///w{self.rank}/seg{i % 2}", 8192 * i, i, 1))
            self.reserved.append(k)
        return out, 0

    def commit(self, keys):
        self.committed += list(keys)

    def abort(self, keys):
        self.aborted += list(keys)


class _Store:
    """Stands in for TuttiKVStore: chunk i of rank r sits in slot i of r's files."""

    def __init__(self, rank, keys):
        self.rank = rank
        self._pool = (None, 100 + rank, 64)
        self.objects = _Objects({k: (f"file:///r{rank}/seg{i % 2}", 4096 * i, i, 1) for i, k in enumerate(keys)},
                                rank)
        self.calls = []
        self.writes = []
        self.fail_writes = False

    def write_placements(self, todo, blocks, mems, stream=None):
        if self.fail_writes:
            raise OSError("injected write failure")
        self.writes.append((list(todo), blocks.tolist(), [int(m) for m in mems]))

        class _Done:
            def wait(self):
                return None

        return _Done()

    def register_peer_pool(self, ptr, nbytes, device):
        return 1000 + device

    def restore_placements(self, todo, blocks, mems=None, layers=None, stream=None, chunk_layer_mems=None):
        if chunk_layer_mems is not None:
            self.calls.append((list(todo), blocks.tolist(), chunk_layer_mems.tolist(), layers))
        else:
            self.calls.append((list(todo), blocks.tolist(), [int(m) for m in mems]))
        return "completion"


class _Peers:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world
        self.ptrs = [0x1000 * (r + 1) for r in range(world)]
        self.nbytes = [1 << 20] * world
        self.devices = list(range(world))


def _fanout_rank_q(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        keys = [bytes([i]) * 16 for i in range(4)]
        store = _Store(rank, keys)
        fan = FanoutRestorer(store, _Peers(rank, world))
        items = [RestoreItem(rank=r, key=k, block_ids=[10 * r + i, 10 * r + i + 1]) for r in range(world)
                 for i, k in enumerate(keys)]
        # slot i lives on drive i % 2; drive d belongs to GPU d
        comp = fan.restore(items, n_drives=2, affine_gpus=[0, 1])
        # replicated cache: rank 0 owns every chunk, all ranks receive it
        rep = [RestoreItem(rank=r, key=k, block_ids=[r, i], source=0) for r in range(world) for i, k in enumerate(keys)]
        comp2 = fan.restore(rep, n_drives=2, affine_gpus=[0, 1])
        q.put((rank, (comp, comp2, store.calls)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _per_layer_rank_q(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from tutti_b200.integration.vllm.worker import fanout_items

        keys = [bytes([i]) * 16 for i in range(4)]
        store = _Store(rank, keys)
        fan = FanoutRestorer(store, _Peers(rank, world))
        # vLLM's per-layer caches: layer l of rank r registered as handle 500 + 10 r + l
        fan.mems, fan.layer_mems = None, [np.asarray([500 + 10 * r + l for l in range(3)], dtype=np.uint64)
                                          for r in range(world)]
        blocks = np.arange(8, dtype=np.int64)
        sliced = fanout_items(keys, blocks, 2, [(r,) for r in range(world)])
        fan.restore(sliced, n_drives=2, affine_gpus=[0, 1], layers=[1])
        shared = fanout_items(keys, blocks, 2, [tuple(range(world))] * world)  # an MLA latent cache
        fan.restore(shared, n_drives=2, affine_gpus=[0, 1], layers=[2])
        q.put((rank, store.calls))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_per_layer_fanout_is_one_submission_and_replicas_share_a_placement():
    out = _spawn(_per_layer_rank_q, 2)
    keys = [bytes([i]) * 16 for i in range(4)]
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        (todo, blocks, clm, layers), (rtodo, rblocks, rclm, rlayers) = out[r]
        # sliced: GPU r reads slots {r, r+2} of both ranks' files in ONE submission; row i holds the
        # per-layer caches of the rank item i lands in
        assert todo == [(f"/r{o}/seg{i % 2}", 4096 * i) for o in range(2) for i in (r, r + 2)]
        assert clm == [[500 + 10 * o + l for l in range(3)] for o in range(2) for _ in (r, r + 2)]
        assert blocks == [[2 * i, 2 * i + 1] for _ in range(2) for i in (r, r + 2)] and layers == [1]
        # replicated: each chunk's owner holds it; both ranks' items name the owner's placement, so
        # the data path reads it once and stores it into both ranks' caches
        owners = [int.from_bytes(k[:8], "little") % 2 for k in keys]
        mine = [i for i, k in enumerate(keys) if i % 2 == r]  # slot i sits on drive i % 2 -> GPU i % 2
        assert rtodo == [(f"/r{owners[i]}/seg{i % 2}", 4096 * i) for _ in range(2) for i in mine]
        assert rclm == [[500 + 10 * o + l for l in range(3)] for o in range(2) for _ in mine] and rlayers == [2]


def test_fanout_items_follow_replica_groups():
    from tutti_b200.integration.vllm.worker import fanout_items
    from tutti_b200.parallel.replica_layout import replica_group, replica_owner

    keys = [bytes([i, 7]) * 8 for i in range(3)]
    blocks = np.arange(6)
    groups = [replica_group(r, 4, 2) for r in range(4)]  # 2 KV heads over TP4: pairs (0,1), (2,3)
    items = fanout_items(keys, blocks, 2, groups)
    assert len(items) == 12
    for it in items:
        g = groups[it.rank]
        assert it.src == replica_owner(it.key, g) and it.src in g
        i = keys.index(it.key)
        assert list(it.block_ids) == [2 * i, 2 * i + 1]
    sliced = fanout_items(keys, blocks, 2, [(r,) for r in range(4)])
    assert all(it.src == it.rank and it.source is None for it in sliced)


def _spawn(fn, world=2, *extra):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=fn, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=30)
    return out


def _store_rank(rank, world, port, q, failing_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        keys = [bytes([i]) * 16 for i in range(4)]
        store = _Store(rank, keys)
        store.fail_writes = rank == failing_rank
        fan = FanoutRestorer(store, _Peers(rank, world))
        items = [RestoreItem(rank=r, key=k, block_ids=[10 * r + i, 10 * r + i + 1]) for r in range(world)
                 for i, k in enumerate(keys)]
        try:
            n = fan.store(items, n_drives=2, affine_gpus=[0, 1])
            res = ("ok", n)
        except RuntimeError as e:
            res = ("error", str(e))
        o = store.objects
        q.put((rank, (res, store.writes, o.committed, o.aborted)))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_fanin_store_writes_drive_affine_share_and_commits_own_keys():
    out = _spawn(_store_rank, 2, -1)
    keys = [bytes([i]) * 16 for i in range(4)]
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        res, writes, committed, aborted = out[r]
        assert res == ("ok", 4)
        # GPU r writes slots {r, r+2} of BOTH ranks' namespaces, gathering from the owner's pool
        todo, blocks, mems = writes[0]
        assert todo == [(f"/w{o}/seg{i % 2}", 8192 * i) for o in range(2) for i in (r, r + 2)]
        assert mems == [100 + r if o == r else 1000 + o for o in range(2) for _ in (r, r + 2)]
        assert blocks == [[10 * o + i, 10 * o + i + 1] for o in range(2) for i in (r, r + 2)]
        assert committed == keys and aborted == []


def test_fanin_store_failure_on_one_gpu_aborts_every_rank():
    out = _spawn(_store_rank, 2, 1)
    keys = [bytes([i]) * 16 for i in range(4)]
    for r in range(2):
        res, _writes, committed, aborted = out[r]
        assert res[0] == "error" and committed == [] and aborted == keys
    assert "injected write failure" in out[1][0][1]
    assert "peer" in out[0][0][1]


def test_fanout_selects_drive_affine_share_for_all_ranks():
    out = _spawn(_fanout_rank_q, 2)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        comp, comp2, calls = out[r]
        assert comp == comp2 == "completion"
        todo, blocks, mems = calls[0]
        # GPU r reads slots {r, r+2} of BOTH ranks' files and lands each in its owner's pool
        want = [(f"/r{o}/seg{i % 2}", 4096 * i) for o in range(2) for i in (r, r + 2)]
        assert todo == want
        assert mems == [100 + r if o == r else 1000 + o for o in range(2) for _ in (r, r + 2)]
        assert blocks == [[10 * o + i, 10 * o + i + 1] for o in range(2) for i in (r, r + 2)]
        rtodo, _rblocks, rmems = calls[1]
        # one placement (rank 0's file) per destination rank: the data path merges them into one read
        assert rtodo == [(f"/r0/seg{i % 2}", 4096 * i) for o in range(2) for i in (r, r + 2)]
        assert rmems == [100 + r if o == r else 1000 + o for o in range(2) for _ in (r, r + 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("mode,store", [("tp", "local"), ("mla", "local"), ("tp", "fanout")])
def test_two_gpu_fanout_restore_matches_local(tmp_path, mode, store):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(port),
           "-m", "tutti_b200.benchmarks.fanout", "--mode", mode, "--prefix-tokens", "4096", "--steps", "2",
           "--warmup", "1", "--root", str(tmp_path / "fan"), "--leases", "32", "--ctas", "16", "--store", store]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=460)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    import json

    res = json.loads(line)
    assert res["ok"] and res["results"]["fanout"]["verified"] and res["results"]["local"]["verified"]


@pytest.mark.gpu
def test_ready_wait_returns_when_the_flag_is_set_and_reports_a_flag_that_never_is():
    """One GPU: a wait on words already at the value passes at once; a wait on a word that
    nothing sets gives up at its deadline, reports it, and the stream goes on."""
    from tutti_b200 import ops

    board = torch.zeros(4, dtype=torch.int64, device="cuda")
    status = torch.full((2,), -1, dtype=torch.int32).pin_memory()
    board[:2] = 7
    ops.ready_wait(board.data_ptr(), 2, 7, 2_000_000_000, status[0:1])
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    # word 3 stays 0: the wait expires after 50 ms with word 1 of [2, 3] missing
    after = torch.zeros(1, device="cuda")
    ops.ready_wait(board.data_ptr() + 16, 2, 1, 50_000_000, status[1:2])
    after.fill_(1.0)  # work behind the expired wait still runs
    torch.cuda.synchronize()
    assert int(status[1]) == 0b11 and float(after) == 1.0
    # a signal stores the value into each target word
    targets = torch.tensor([board.data_ptr() + 16, board.data_ptr() + 24], dtype=torch.int64, device="cuda")
    ops.ready_signal(targets, 9)
    torch.cuda.synchronize()
    assert board.tolist() == [7, 7, 9, 9]


def _replica_io_worker_rank(rank, world, port, q, root, saves="local"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from tutti_b200.integration.vllm.factory import ConnectorConfig, make_engine
        from tutti_b200.integration.vllm.metadata import LoadSpec, SaveSpec, TuttiConnectorMetadata
        from tutti_b200.integration.vllm.worker import WorkerSide

        bs, chunk, nl, nb = 16, 64, 4, 128
        cfg = ConnectorConfig.from_extra({
            "chunk_tokens": chunk, "replica_io": True,
            "store": {"type": "tutti", "root": f"{root}/r{{RANK}}",
                      "mounts": [f"{root}/nvme0", f"{root}/nvme1"], "capacity_chunks": 64,
                      "segment_file_slots": 16,
                      "runtime_options": {"leases": 16, "max_ctas_per_op": 8, "emulator_media": "memory",
                                          "image_budget_bytes": 256 << 20}}})
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        # this rank's KV-head slice: different values on every rank
        layers = [torch.randn(2, nb, bs, 2, 128, device="cuda", generator=g, dtype=torch.bfloat16) for _ in range(nl)]
        w = WorkerSide(lambda t, entity="": make_engine(cfg, t, rank, rank, world, entity), block_size=bs,
                       chunk_tokens=chunk, tp_rank=rank, tp_size=world, replica_io=True, group=dist.group.WORLD,
                       replica_io_saves=saves)
        w.register_kv_caches({f"model.layers.{i}.self_attn.attn": t for i, t in enumerate(layers)})
        assert w._fan is not None, "replica_io was not set up"
        keys = [bytes([i + 1]) * 16 for i in range(6)]
        src = list(range(0, 24))  # 6 chunks x 4 blocks
        committed = dict(w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", keys, src)])).committed)
        # vLLM's scheduler loads a chunk only once every TP rank reported it committed
        if saves == "fanin":
            for step in range(2, 2000):  # every rank decides a batch at the same call
                if len(committed) == len(keys):
                    break
                committed.update(w.wait_for_save(TuttiConnectorMetadata(step, [], [])).committed)
            assert len(committed) == len(keys), committed
        else:
            assert w.settle_saves() == 1
        dist.barrier()
        ref = [t[:, 0:24].clone() for t in layers]
        dst = list(range(64, 88))
        for t in layers:
            t[:, 64:88].zero_()
        meta = TuttiConnectorMetadata(3, [LoadSpec("b", keys, dst, len(keys) * chunk)], [])
        w.start_load_kv(meta)
        for i in range(nl):
            w.wait_for_layer_load(f"model.layers.{i}.self_attn.attn")
        wm = w.wait_for_save(meta)
        torch.cuda.synchronize()
        ok = all(torch.equal(layers[i][:, 64:88], ref[i]) for i in range(nl))
        stats = w.engine.store.runtime.controller_stats()
        q.put((rank, (ok, dict(wm.failed_loads), sum(s["read_bytes"] for s in stats))))
        dist.barrier()
        w.shutdown()
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, "".join(traceback.format_exception(e))[-3000:]))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("saves", ["local", "fanin"])
def test_two_gpu_vllm_worker_with_replica_io_restores_every_rank(tmp_path, saves):
    """replica_io in the vLLM worker: each GPU reads the chunks on its affine drive for both
    ranks, its io kernel stores each rank's slice into that rank's per-layer caches over NVLink,
    and every layer's attention waits on device-side ready flags from both ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = _spawn(_replica_io_worker_rank, 2, str(tmp_path), saves)
    for r in range(2):
        assert isinstance(out[r], tuple), out[r]
        ok, failed, read_bytes = out[r]
        assert ok and failed == {}
    # drive-affine: each GPU read part of the chunks (for both ranks), none read them all
    assert all(out[r][2] > 0 for r in range(2))


class _Comp:
    def __init__(self, fail=False):
        self.done, self.fail = False, fail

    def query(self):
        return self.done

    def wait(self):
        if self.fail:
            raise OSError("injected write failure")


class _Board:
    """ReadyBoard stand-in: waits are tickets whose outcome the test decides."""

    def __init__(self):
        self.signals, self.waits = [], []
        self.gave_up = set()

    def signal(self, slot, value, stream=None):
        self.signals.append((slot, value))

    def wait(self, slot, value, stream=None, timeout_s=10.0):
        self.waits.append((slot, value))
        return len(self.waits) - 1

    def passed(self, t):
        return True

    def failed(self, t):
        return [1] if t in self.gave_up else []

    def close(self):
        pass


def _fanin_rank(rank, world, port, q, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from types import SimpleNamespace

        from tutti_b200.integration.vllm.metadata import SaveSpec, TuttiConnectorMetadata
        from tutti_b200.integration.vllm.worker import WorkerSide

        keys = [bytes([i]) * 16 for i in range(4)]
        more = [bytes([i]) * 16 for i in range(4, 6)]
        store = _Store(rank, [])
        store.objects.reserved = []
        comps = []

        def write_placements(todo, blocks, mems=None, stream=None, chunk_layer_mems=None):
            if rank == fail_rank and len(comps) == 1:
                raise OSError("injected write failure")
            store.writes.append((list(todo), blocks.tolist(), chunk_layer_mems.tolist()))
            comps.append(_Comp())
            return comps[-1]

        store.write_placements = write_placements
        fan = FanoutRestorer(store, _Peers(rank, world))
        fan.mems, fan.layer_mems = None, [np.asarray([500 + 10 * r + l for l in range(2)], dtype=np.uint64)
                                          for r in range(world)]
        confirmed = []
        index = SimpleNamespace(confirm_store=lambda ks, ok: confirmed.append((list(ks), ok)),
                                is_resident=lambda k: False)
        engine = SimpleNamespace(plan_store=lambda ks: SimpleNamespace(new_keys=list(ks)), index=index,
                                 write_stream=None, staged=False, store=store)
        w = WorkerSide(lambda t: None, block_size=16, chunk_tokens=32, tp_rank=rank, tp_size=world,
                       replica_io=True, replica_io_saves="fanin")
        board = _Board()
        w.engine, w._fan, w._save_board, w._fanin_on = engine, fan, board, True
        w._n_drives, w._affine = 2, [0, 1]
        out = {}
        # step 1: four chunks saved; this GPU writes the chunks on its drive for both ranks
        m1 = w.wait_for_save(TuttiConnectorMetadata(1, [], [SaveSpec("a", keys, list(range(8)))]))
        out["step1_committed"] = dict(m1.committed)
        out["writes"] = store.writes[0]
        out["signals"] = list(board.signals)
        # step 2: request a finished: its next forward waits for every GPU's writes of batch 1
        w.start_load_kv(TuttiConnectorMetadata(2, [], [], finished_saving=["a"]))
        out["reuse_waits"] = [x for x in board.waits if x[0] == 1]
        m2 = w.wait_for_save(TuttiConnectorMetadata(2, [], []))  # writes still running: undecided
        out["step2_committed"] = dict(m2.committed)
        comps[0].done = True
        w.start_load_kv(TuttiConnectorMetadata(3, [], []))
        m3 = w.wait_for_save(TuttiConnectorMetadata(3, [], [SaveSpec("b", more, list(range(8, 12)))]))
        out["step3_committed"] = sorted(m3.committed)
        for c in comps:
            c.done = True
        w.start_load_kv(TuttiConnectorMetadata(4, [], []))
        m4 = w.wait_for_save(TuttiConnectorMetadata(4, [], []))
        out["step4_committed"] = sorted(m4.committed)
        out["objects"] = (list(store.objects.committed), list(store.objects.aborted))
        out["confirmed"] = confirmed
        out["pending"] = len(w._fanin)
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, "".join(traceback.format_exception(e))[-3000:]))
    finally:
        dist.destroy_process_group()


def test_fanin_saves_commit_together_after_every_gpu_wrote():
    out = _spawn(_fanin_rank, 2, -1)
    keys = [bytes([i]) * 16 for i in range(4)]
    more = [bytes([i]) * 16 for i in range(4, 6)]
    for r in range(2):
        o = out[r]
        assert not isinstance(o, str), o
        todo, blocks, clm = o["writes"]
        # GPU r writes slots {r, r+2} of both ranks' namespaces, gathering from each owner's caches
        assert todo == [(f"/w{owner}/seg{i % 2}", 8192 * i) for owner in range(2) for i in (r, r + 2)]
        assert clm == [[500 + 10 * owner + l for l in range(2)] for owner in range(2) for _ in (r, r + 2)]
        assert blocks == [[2 * i, 2 * i + 1] for _ in range(2) for i in (r, r + 2)]
        assert (0, 1) in o["signals"] and (1, 1) in o["signals"]  # forward done, writes done
        assert o["reuse_waits"] == [(1, 1)]
        assert o["step1_committed"] == {} and o["step2_committed"] == {}
        assert o["step3_committed"] == sorted(keys)  # batch 1 decided once both GPUs' writes ended
        assert o["step4_committed"] == sorted(more)
        committed, aborted = o["objects"]
        assert committed == keys + more and aborted == [] and o["pending"] == 0
        assert (keys, True) in o["confirmed"] and (more, True) in o["confirmed"]


def test_fanin_save_failure_on_one_gpu_aborts_the_batch_on_every_rank():
    out = _spawn(_fanin_rank, 2, 1)  # GPU 1's second batch fails to submit
    keys = [bytes([i]) * 16 for i in range(4)]
    more = [bytes([i]) * 16 for i in range(4, 6)]
    for r in range(2):
        o = out[r]
        assert not isinstance(o, str), o
        committed, aborted = o["objects"]
        assert committed == keys and aborted == more
        assert o["step4_committed"] == [] and (more, False) in o["confirmed"] and o["pending"] == 0


def _fanin_pressure_rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from types import SimpleNamespace

        from tutti_b200.integration.vllm.metadata import SaveSpec, TuttiConnectorMetadata
        from tutti_b200.integration.vllm.worker import WorkerSide

        store = _Store(rank, [])
        comps = []

        def write_placements(todo, blocks, mems=None, stream=None, chunk_layer_mems=None):
            comps.append(_Comp())  # never reports done on its own: only a blocking wait settles it
            return comps[-1]

        store.write_placements = write_placements
        fan = FanoutRestorer(store, _Peers(rank, world))
        fan.mems, fan.layer_mems = None, [np.zeros(2, dtype=np.uint64) for _ in range(world)]
        index = SimpleNamespace(confirm_store=lambda ks, ok: None, is_resident=lambda k: False)
        engine = SimpleNamespace(plan_store=lambda ks: SimpleNamespace(new_keys=list(ks)), index=index,
                                 write_stream=None, staged=False, store=store)
        w = WorkerSide(lambda t: None, block_size=16, chunk_tokens=32, tp_rank=rank, tp_size=world,
                       replica_io=True, replica_io_saves="fanin", max_inflight_saves=1)
        w.engine, w._fan, w._save_board, w._fanin_on = engine, fan, _Board(), True
        w._n_drives, w._affine = 2, [0, 1]
        sizes = []
        for step in range(3):
            keys = [bytes([10 * step + i]) * 16 for i in range(2)]
            w.wait_for_save(TuttiConnectorMetadata(step + 1, [], [SaveSpec(f"r{step}", keys, [0, 1, 2, 3])]))
            sizes.append(len(w._fanin))
        q.put((rank, (sizes, len(store.objects.committed))))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, "".join(traceback.format_exception(e))[-3000:]))
    finally:
        dist.destroy_process_group()


def test_fanin_saves_back_pressure_decides_every_batch_when_too_many_wait():
    out = _spawn(_fanin_pressure_rank, 2)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        sizes, committed = out[r]
        # one batch may stay undecided; the second forces a blocking harvest that decides both
        assert sizes == [1, 0, 1] and committed == 4
