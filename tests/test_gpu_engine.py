"""KV engine on the GPU: layerwise restore overlapped with prefill equals a full recompute."""
import numpy as np
import pytest
import torch

from tutti_b200.engine.core import KVEngine
from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.models.llama import LlamaConfig, LlamaModel
from tutti_b200.storage.memory import MemoryKVStore
from tutti_b200.storage.tutti_store import TuttiKVStore

pytestmark = pytest.mark.gpu

CFG = LlamaConfig(hidden=256, layers=3, heads=4, kv_heads=2, head_dim=64, intermediate=512, vocab=1000)


def setup(tmp_path, staged=False):
    g = CFG.geometry(block_size=16, chunk_tokens=64)
    if staged:
        store = MemoryKVStore(g.chunk_bytes, capacity_chunks=64)
        store.open()
    else:
        store = TuttiKVStore(tmp_path, g, capacity_chunks=64, mounts=[str(tmp_path / "nvme0")], device=0,
                             segment_file_slots=16, runtime_options={"leases": 16, "max_ctas_per_op": 4})
        store.open()
    model = LlamaModel(CFG, "cuda", seed=1)
    pool = torch.zeros(g.pool_shape(128), dtype=torch.bfloat16, device="cuda")
    eng = KVEngine(store, g, device=0)
    eng.bind(pool)
    return g, store, model, pool, eng


@pytest.mark.parametrize("staged", [False, True])
def test_layerwise_restore_then_prefill_matches_recompute(tmp_path, staged):
    g, store, model, pool, eng = setup(tmp_path, staged)
    try:
        rng = np.random.default_rng(0)
        P, N = 256, 32
        prompts = [torch.from_numpy(rng.integers(0, CFG.vocab, size=P + N)) for _ in range(2)]
        nbr = (P + N + 15) // 16
        tables = [torch.arange(r * nbr, (r + 1) * nbr) for r in range(2)]
        full = model.prefill(prompts, [0, 0], tables, pool)  # reference: no reuse
        for r in range(2):
            keys = chunk_keys_for_tokens(prompts[r][:P].tolist(), 64)
            comp = eng.store_chunks(keys, tables[r][: P // 16])
            comp.wait()
        eng.wait_idle()
        # fresh placement
        pool.zero_()
        perm = torch.randperm(128)[: 2 * nbr]
        t2 = [perm[:nbr], perm[nbr:]]
        keys, hits = [], []
        for r in range(2):
            k = chunk_keys_for_tokens(prompts[r][:P].tolist(), 64)
            hits.append(eng.lookup_prefix_keys(k))
            keys += k
        assert hits == [P, P]
        table = torch.cat([t2[r][: P // 16] for r in range(2)])
        news = [prompts[r][P:] for r in range(2)]
        if staged:
            eng.load(keys, table).wait()
            out = model.prefill(news, hits, t2, pool)
        else:
            plan = eng.start_read_plan(keys, table, window=2)
            out = model.prefill(news, hits, t2, pool, wait_layer=plan.wait_layer)
            plan.finish()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), full.float(), atol=3e-2, rtol=3e-2)
    finally:
        store.close()


def test_writes_on_their_own_stream_overlap_reads(tmp_path):
    """defer_writes_after_reads=False: a store on the write stream runs beside a restore on the IO stream."""
    g = CFG.geometry(block_size=16, chunk_tokens=64)
    store = TuttiKVStore(tmp_path, g, capacity_chunks=64, mounts=[str(tmp_path / "nvme0")], device=0,
                         segment_file_slots=16, runtime_options={"leases": 16, "max_ctas_per_op": 4})
    store.open()
    try:
        pool = torch.randn(g.pool_shape(128), device="cuda").to(torch.bfloat16)
        eng = KVEngine(store, g, device=0, defer_writes_after_reads=False)
        eng.bind(pool)
        assert eng.write_stream is not eng.io_stream
        keys_a = chunk_keys_for_tokens(list(range(256)), 64)
        keys_b = chunk_keys_for_tokens(list(range(1000, 1256)), 64)
        ta, tb, ta2, tb2 = (torch.arange(s, s + 16) for s in (0, 16, 32, 48))
        eng.store_chunks(keys_a, ta).wait()
        read = eng.load(keys_a, ta2)  # IO stream
        write = eng.store_chunks(keys_b, tb)  # write stream, concurrently
        read.wait()
        write.wait()
        eng.wait_idle()
        torch.cuda.synchronize()
        assert torch.equal(pool[:, :, ta2], pool[:, :, ta])
        eng.load(keys_b, tb2).wait()
        torch.cuda.synchronize()
        assert torch.equal(pool[:, :, tb2], pool[:, :, tb])
    finally:
        store.close()
