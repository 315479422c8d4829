import hashlib
import struct

import pytest

from tutti_b200.index.chunk_index import (IO_KEY_BYTES, ChunkIndex, chunk_digest, chunk_key_of,
                                          chunk_keys_for_tokens, decode_io_key, derive_io_key, layer_of)


def ref_key(parent, toks):
    return hashlib.blake2b(parent + b"".join(struct.pack("<Q", t) for t in toks), digest_size=16).digest()


def test_key_chain_matches_blake2b_definition():
    toks = list(range(1000, 1000 + 64 * 3 + 5))
    keys = chunk_keys_for_tokens(toks, 64, namespace=b"ns")
    assert len(keys) == 3
    p = b"ns"
    for i, k in enumerate(keys):
        p = ref_key(p, toks[i * 64:(i + 1) * 64])
        assert k == p


def test_io_key_roundtrip():
    k = chunk_digest(b"", [1, 2, 3])
    io = derive_io_key(k, 513)
    assert len(io) == IO_KEY_BYTES
    assert chunk_key_of(io) == k and layer_of(io) == 513
    assert decode_io_key(io) == (k, 513)
    with pytest.raises(ValueError):
        derive_io_key(k, 1 << 16)
    with pytest.raises(ValueError):
        layer_of(b"short")


def test_plan_confirm_lookup_and_lru_eviction():
    idx = ChunkIndex(capacity=3, chunk_tokens=4)
    toks = list(range(12))
    keys, _ = idx.hash_keys(toks)
    plan = idx.plan_store(keys)
    assert plan.new_keys == keys and plan.evicted_keys == []
    assert idx.lookup_prefix(toks) == 0  # pending never hits
    idx.confirm_store(keys)
    assert idx.lookup_prefix(toks) == 12
    other, _ = idx.hash_keys(list(range(100, 104)))
    idx.pin([keys[1]])
    plan = idx.plan_store(other)
    # oldest unpinned resident goes first; keys[0] was refreshed by lookup order -> keys[0] oldest
    assert plan.evicted_keys == [keys[0]]
    idx.confirm_store(other)
    assert not idx.is_resident(keys[0]) and idx.is_resident(keys[1])
    assert idx.plan_store(other) is not None  # all resident -> nothing new
    idx.unpin([keys[1]])
    with pytest.raises(KeyError):
        idx.unpin([keys[1]])


def test_pending_duplicate_rejected_and_stale_reclaim():
    idx = ChunkIndex(capacity=4, chunk_tokens=2)
    keys, _ = idx.hash_keys([1, 2, 3, 4])
    assert idx.plan_store(keys) is not None
    assert idx.plan_store(keys) is None
    for _ in range(5):
        idx.advance_epoch()
    assert sorted(idx.reclaim_stale_pending(3)) == sorted(keys)
    assert idx.stats()["pending"] == 0


def test_incremental_hash_matches_full():
    idx = ChunkIndex(capacity=10, chunk_tokens=8, namespace=b"m")
    toks = list(range(40))
    full, last = idx.hash_keys(toks)
    a, p = idx.hash_keys(toks[:16])
    b, p2 = idx.hash_keys(toks, start=16, parent=p)
    assert a + b == full and p2 == last


def test_eviction_picks_the_coldest_unpinned_key_among_many_pinned():
    idx = ChunkIndex(capacity=200, chunk_tokens=1)
    keys = [bytes([i // 256, i % 256]) * 8 for i in range(200)]
    assert idx.plan_store(keys) is not None
    idx.confirm_store(keys)
    idx.pin(keys[:150])  # the 150 coldest are pinned
    idx.mark_recent(keys[160:])  # keys[150:160] are now the coldest unpinned ones
    new = [b"\xff" * 16, b"\xfe" * 16]
    plan = idx.plan_store(new)
    assert plan.evicted_keys == keys[150:152]
    assert idx.stats() == {"capacity": 200, "resident": 198, "pending": 2, "pinned": 150, "epoch": 0}
    # a deficit the unpinned keys cannot cover is refused without a change
    idx.pin(keys[152:])
    assert idx.plan_store([bytes([7]) * 16]) is None
    assert idx.stats()["resident"] == 198


def test_lookup_many_matches_lookup_prefix():
    idx = ChunkIndex(capacity=16, chunk_tokens=4, namespace=b"ns")
    prompts = [list(range(10)), list(range(100, 117)), list(range(3))]
    keys, _ = idx.hash_keys(prompts[0])
    idx.plan_store(keys)
    idx.confirm_store(keys)
    hits = idx.lookup_many(prompts)
    assert [h for h, _ in hits] == [8, 0, 0]
    assert hits[0][1] == keys and len(hits[1][1]) == 4 and hits[2][1] == []
    assert [idx.lookup_prefix(p) for p in prompts] == [8, 0, 0]
