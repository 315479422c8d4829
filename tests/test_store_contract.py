"""One KV-engine contract over two stores: the staged in-memory store and the direct segment-file store.

The segment-file store runs on the POSIX backend here (host pread/pwrite straight
into a host-memory pool), so the direct paged path is exercised without a GPU.
Parity: reference tests/python/storage/test_store_contract.py (one contract, Memory and Tutti stores).
"""
import numpy as np
import pytest
import torch

from tutti_b200.engine.core import KVEngine
from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.models.kv_geometry import KVGeometry
from tutti_b200.storage.memory import MemoryKVStore
from tutti_b200.storage.tutti_store import TuttiKVStore

G = KVGeometry("contract", num_layers=2, num_kv_heads=2, head_dim=64, block_size=16, chunk_tokens=32)
CAP = 6


def open_store(kind, root):
    if kind == "memory":
        s = MemoryKVStore(G.chunk_bytes, capacity_chunks=CAP)
        s.open()
        return s
    return TuttiKVStore(root, G, capacity_chunks=CAP, mounts=[str(root / "m0"), str(root / "m1")], backend="posix",
                        device=-1, segment_file_slots=4, runtime_options={"threads": 2, "direct_io": False}).open()


@pytest.fixture(params=["memory", "segment-files"])
def env(request, tmp_path):
    store = open_store(request.param, tmp_path)
    eng = KVEngine(store, G, capacity_chunks=CAP, device=torch.device("cpu"))
    pool = torch.randn(G.pool_shape(64)).to(torch.bfloat16)
    eng.bind(pool)
    yield request.param, store, eng, pool, tmp_path
    store.close()


def keys_for(i, n=1):
    return chunk_keys_for_tokens(list(range(i * 1000, i * 1000 + 32 * n)), 32)


def test_roundtrip_to_other_blocks(env):
    kind, store, eng, pool, _ = env
    k = keys_for(0, 3)
    eng.store_chunks(k, torch.arange(0, 6)).wait()
    assert eng.lookup_prefix_keys(k) == 96
    ref = pool[:, :, 0:6].clone()
    eng.load(k, torch.tensor([40, 41, 50, 51, 60, 61])).wait()
    got = pool[:, :, torch.tensor([40, 41, 50, 51, 60, 61])]
    assert torch.equal(got, ref)
    assert eng.store_chunks(k, torch.arange(0, 6)) is None  # resident chunks are not written again


def test_capacity_closure_evicts_lru_but_never_pinned(env):
    kind, store, eng, pool, _ = env
    chunks = [keys_for(i) for i in range(CAP)]
    for i, k in enumerate(chunks):
        eng.store_chunks(k, torch.arange(2 * i, 2 * i + 2)).wait()
    eng.pin(chunks[0])
    eng.store_chunks(keys_for(100), torch.arange(20, 22)).wait()  # full: evicts the oldest unpinned
    assert eng.lookup_prefix_keys(chunks[0]) == 32 and eng.lookup_prefix_keys(chunks[1]) == 0
    ref = pool[:, :, 0:2].clone()
    eng.load(chunks[0], torch.arange(30, 32)).wait()
    assert torch.equal(pool[:, :, 30:32], ref)
    with pytest.raises(Exception):  # the evicted chunk is gone from the store too
        eng.load(chunks[1], torch.arange(32, 34)).wait()
    eng.unpin(chunks[0])


def test_a_fresh_engine_finds_persisted_chunks(env):
    kind, store, eng, pool, root = env
    k = keys_for(7, 2)
    eng.store_chunks(k, torch.arange(4, 8)).wait()
    eng.wait_idle()
    if kind == "memory":
        pytest.skip("the in-memory store does not outlive its process")
    ref = pool[:, :, 4:8].clone()
    store.objects.checkpoint()
    store.close()
    store2 = open_store(kind, root)
    try:
        eng2 = KVEngine(store2, G, capacity_chunks=CAP, device=torch.device("cpu"))
        pool2 = torch.zeros(G.pool_shape(64), dtype=torch.bfloat16)
        eng2.bind(pool2)
        assert eng2.restore_from_store() == 2 and eng2.lookup_prefix_keys(k) == 64
        eng2.load(k, torch.arange(10, 14)).wait()
        assert torch.equal(pool2[:, :, 10:14], ref)
    finally:
        store2.close()


def test_layerwise_plan_on_a_host_pool(env):
    kind, store, eng, pool, _ = env
    if kind == "memory":
        pytest.skip("layerwise plans need a direct store")
    k = keys_for(3, 2)
    eng.store_chunks(k, torch.arange(0, 4)).wait()
    ref = pool[:, :, 0:4].clone()
    plan = eng.start_read_plan(k, torch.arange(20, 24))
    for layer in range(G.num_layers):
        plan.wait_layer(layer)
    plan.finish()
    assert torch.equal(pool[:, :, 20:24], ref) and plan.read_ms() is not None


def test_one_placement_restore_lands_in_several_ranks_per_layer_caches(tmp_path):
    """chunk_layer_mems: row i names the per-layer caches of the rank item i lands in; a placement
    named for two ranks (a replicated cache) is read once and stored into both."""
    store = open_store("segment-files", tmp_path)
    try:
        gen = torch.Generator().manual_seed(5)
        own = [torch.randn(G.planes, 32, G.block_size, G.num_kv_heads, G.head_dim, generator=gen).to(torch.bfloat16)
               for _ in range(G.num_layers)]
        store.register_layers(own)
        k = keys_for(7, 2)
        store.put_paged(k, np.arange(4).reshape(2, 2)).wait()
        peer = [torch.zeros_like(t) for t in own]  # another rank's per-layer caches
        peer_h = [store.runtime.register_memory(t.data_ptr(), t.numel() * t.element_size(), "host", -1) for t in peer]
        own_h = [int(h) for h in store._layer_mems]
        places = []
        for key in k:
            uri, off, _slot, _gen = store.objects.lookup(bytes(key))
            places.append((uri[len("file://"):], off))
        # chunk 0 for both ranks (same placement twice), chunk 1 for the peer only
        todo = [places[0], places[0], places[1]]
        blocks = np.asarray([[10, 11], [20, 21], [22, 23]], dtype=np.int64)
        clm = np.asarray([own_h, peer_h, peer_h], dtype=np.uint64)
        store.restore_placements(todo, blocks, chunk_layer_mems=clm).wait()
        for l in range(G.num_layers):
            assert torch.equal(own[l][:, 10:12], own[l][:, 0:2])
            assert torch.equal(peer[l][:, 20:22], own[l][:, 0:2])
            assert torch.equal(peer[l][:, 22:24], own[l][:, 2:4])
        with pytest.raises(ValueError, match="chunk_layer_mems"):
            store.restore_placements(todo, blocks, chunk_layer_mems=clm[:2])
    finally:
        store.close()


def test_one_write_submission_gathers_from_several_ranks_per_layer_caches(tmp_path):
    """write_placements with chunk_layer_mems: chunk i is gathered from the per-layer caches row i names
    (the fan-in store's single submission for every owner), then read back and compared."""
    store = open_store("segment-files", tmp_path)
    try:
        gen = torch.Generator().manual_seed(9)
        shape = (G.planes, 16, G.block_size, G.num_kv_heads, G.head_dim)
        own = [torch.randn(*shape, generator=gen).to(torch.bfloat16) for _ in range(G.num_layers)]
        peer = [torch.randn(*shape, generator=gen).to(torch.bfloat16) for _ in range(G.num_layers)]
        store.register_layers(own)
        peer_h = [store.runtime.register_memory(t.data_ptr(), t.numel() * t.element_size(), "host", -1) for t in peer]
        own_h = [int(h) for h in store._layer_mems]
        keys = keys_for(11, 2)
        accepted, rejected = store.reserve(keys)
        assert rejected == 0
        where = {bytes(k): (uri[len("file://"):], off) for k, uri, off, _slot, _gen in accepted}
        todo = [where[bytes(keys[0])], where[bytes(keys[1])]]
        # chunk 0 from this rank's blocks 0-1, chunk 1 from the peer's blocks 4-5
        store.write_placements(todo, np.asarray([[0, 1], [4, 5]]),
                               chunk_layer_mems=np.asarray([own_h, peer_h], dtype=np.uint64)).wait()
        store.objects.commit([bytes(k) for k in keys])
        store.get_paged(keys, np.asarray([[8, 9], [10, 11]])).wait()
        for l in range(G.num_layers):
            assert torch.equal(own[l][:, 8:10], own[l][:, 0:2])
            assert torch.equal(own[l][:, 10:12], peer[l][:, 4:6])
    finally:
        store.close()
