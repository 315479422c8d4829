"""Staged stores: one reused staging buffer per direction, reuse gated on the previous batch."""
import torch

from tutti_b200.engine.core import KVEngine
from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.models.kv_geometry import KVGeometry
from tutti_b200.storage.base import DoneCompletion
from tutti_b200.storage.memory import MemoryKVStore

G = KVGeometry("t", num_layers=2, num_kv_heads=2, head_dim=64, block_size=16, chunk_tokens=32)


def engine(store):
    eng = KVEngine(store, G, capacity_chunks=256, device=torch.device("cpu"), staged=True)
    pool = torch.randn(G.pool_shape(128)).to(torch.bfloat16)
    eng.bind(pool)
    return eng, pool


def test_repeated_staged_batches_reuse_one_registration_per_direction():
    store = MemoryKVStore(G.chunk_bytes, capacity_chunks=256)
    store.open()
    eng, pool = engine(store)
    ref = pool.clone()
    done = []
    for n, start in [(1, 0), (3, 1), (2, 4), (5, 6), (1, 11), (4, 12)]:
        keys = chunk_keys_for_tokens(list(range(start * 32, (start + n) * 32)), 32)
        eng.store_chunks(keys, torch.arange(2 * start, 2 * (start + n))).wait()
        done.append((keys, start, n))
    pool.zero_()
    for keys, start, n in reversed(done):
        eng.load(keys, torch.arange(64 + 2 * start, 64 + 2 * (start + n))).wait()
        assert torch.equal(pool[:, :, 64 + 2 * start:64 + 2 * (start + n)], ref[:, :, 2 * start:2 * (start + n)])
    assert len(store._buffers) == 2  # one per direction, not one per batch
    assert eng._staging("store").allocations <= 3 and eng._staging("store").capacity_chunks == 8


class LazyStore(MemoryKVStore):
    """A store whose put reads the staging buffer only when the batch is waited on."""

    def put_batch(self, batch):
        store = self

        class Later:
            done = False

            def query(self):
                return self.done

            def wait(self):
                if not self.done:
                    MemoryKVStore.put_batch(store, batch)
                    self.done = True

        return Later()


def test_store_buffer_is_not_reused_before_the_previous_put_completes():
    store = LazyStore(G.chunk_bytes, capacity_chunks=64)
    store.open()
    eng, pool = engine(store)
    ref = pool.clone()
    k1 = chunk_keys_for_tokens(list(range(64)), 32, namespace=b"a")
    k2 = chunk_keys_for_tokens(list(range(64)), 32, namespace=b"b")
    c1 = eng.store_chunks(k1, torch.arange(0, 4))  # not completed yet
    c2 = eng.store_chunks(k2, torch.arange(8, 12))  # must not overwrite batch 1's bytes first
    c1.wait()
    c2.wait()
    pool.zero_()
    eng.load(k1, torch.arange(20, 24)).wait()
    eng.load(k2, torch.arange(30, 34)).wait()
    assert torch.equal(pool[:, :, 20:24], ref[:, :, 0:4])
    assert torch.equal(pool[:, :, 30:34], ref[:, :, 8:12])
    assert isinstance(DoneCompletion(), DoneCompletion)


def test_checkpoint_interval_zero_turns_periodic_checkpoints_off():
    calls = []

    class Objects:
        def checkpoint(self):
            calls.append(1)

    store = MemoryKVStore(G.chunk_bytes, capacity_chunks=8)
    store.open()
    store.objects = Objects()
    off = KVEngine(store, G, capacity_chunks=8, device=torch.device("cpu"), staged=True, checkpoint_interval_s=0)
    off.poll_writes()
    off.wait_idle()
    assert calls == []
    off._maybe_checkpoint(force=True)  # an explicit checkpoint still happens
    assert calls == [1]
    every = KVEngine(store, G, capacity_chunks=8, device=torch.device("cpu"), staged=True, checkpoint_interval_s=1e-9)
    every.poll_writes()
    assert calls == [1, 1]
