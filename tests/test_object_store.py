import os
import struct

import pytest

from tutti_b200._native import core


def cfg(root, **kw):
    c = {"uri": str(root), "segment_bytes": 8192, "segment_count": 3, "segment_file_slots": 4,
         "segment_header_bytes": 131072, "capacity_slots": 16, "fingerprint": "fp-1",
         "mounts": [str(root / "d0"), str(root / "d1")]}
    c.update(kw)
    return c


def test_digests_match_published_check_values():
    c = core()
    assert c.crc32c(b"123456789") == 0xE3069283  # CRC-32C check value
    assert c.crc32c(b"") == 0


def test_slot_placement_matches_segment_file_format(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    slot_bytes = 131072 + 3 * 8192
    assert s.slot_bytes == slot_bytes
    # slot % N picks the device; (slot / N) / slots_per_file the file
    assert s.slot_path(0).endswith("d0/r0/segments/0.seg")
    assert s.slot_path(1).endswith("d1/r0/segments/0.seg")
    assert s.slot_path(9).endswith("d1/r0/segments/1.seg")
    assert s.header_offset_for_slot(5) == (5 // 2 % 4) * slot_bytes
    assert s.payload_offset_for_slot(5) == s.header_offset_for_slot(5) + 131072
    assert s.ready_slots == 8  # first file group materialised at open
    assert os.path.getsize(s.slot_path(0)) == 4 * slot_bytes
    s.close()


def test_reserve_commit_header_and_recover(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    keys = [bytes([i]) * 18 for i in range(5)]
    acc, rej = s.reserve(keys)
    assert rej == 0 and len(acc) == 5
    assert s.contains_prefix(keys) == 0
    s.commit(keys)
    assert s.contains_prefix(keys) == 5
    # header bytes on media
    _, uri, off, slot, gen = acc[2]
    path = uri[len("file://"):]
    with open(path, "rb") as f:
        f.seek(s.header_offset_for_slot(slot))
        h = f.read(4096)
    assert h[:8] == b"TUTTIOBJ"
    assert struct.unpack_from("<I", h, 56)[0] == core().crc32c(h[:56])
    assert struct.unpack_from("<Q", h, 16)[0] == core().object_identity(keys[2])
    assert h[64:64 + 18] == keys[2]
    s.close()
    s2 = core().ObjectStore()
    s2.open(cfg(tmp_path))
    rec = s2.recover()
    assert sorted(rec) == sorted(keys)
    assert s2.lookup(keys[2])[2] == slot
    s2.close()


def test_uncommitted_is_never_written_and_release_invalidates(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    a, b = b"a" * 18, b"b" * 18
    s.reserve([a, b])
    s.commit([a])
    s.pin([a])
    assert s.release([a]) == 0  # pinned
    s.unpin([a])
    assert s.release([a]) == 1
    s.close()
    s2 = core().ObjectStore()
    s2.open(cfg(tmp_path))
    assert s2.recover() == []
    s2.close()


def test_fingerprint_mismatch_fails_closed(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    s.close()
    s2 = core().ObjectStore()
    with pytest.raises(ValueError):
        s2.open(cfg(tmp_path, fingerprint="other"))


def test_capacity_partial_acceptance_and_precreate(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path, capacity_slots=16))
    keys = [bytes([i]) * 18 for i in range(12)]
    acc, rej = s.reserve(keys)
    assert len(acc) == 8 and rej == 4  # only the first group is ready
    assert s.precreate_step(100) == 8
    acc2, rej2 = s.reserve(keys)
    assert rej2 == 0 and len(acc2) == 12
    s.close()


def test_read_only_refuses_mutation(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    s.reserve([b"k" * 18])
    s.commit([b"k" * 18])
    s.close()
    ro = core().ObjectStore()
    ro.open(cfg(tmp_path, read_only=True))
    assert ro.recover() == [b"k" * 18]
    with pytest.raises(RuntimeError):
        ro.reserve([b"z" * 18])
    ro.close()


def test_residency_bitmaps_all_ranks(tmp_path):
    stores = []
    for r in range(2):
        s = core().ObjectStore()
        s.open(cfg(tmp_path, rank_id=r, rank_count=2))
        stores.append(s)
    # reopen rank 0 so it maps rank 1's bitmap
    keys = [b"x" * 18, b"y" * 18]
    for s in stores:
        s.reserve(keys)
    stores[0].commit(keys)
    stores[1].commit(keys[:1])
    stores[0].close()
    s0 = core().ObjectStore()
    s0.open(cfg(tmp_path, rank_id=0, rank_count=2))
    s0.recover()
    assert s0.contains_prefix(keys) == 2
    assert s0.contains_prefix(keys, True) == 1
    s0.close()
    stores[1].close()


def test_stored_geometry_fp8_sizes():
    from tutti_b200.models.kv_geometry import DEEPSEEK_V3_MLA, LLAMA3_8B
    from tutti_b200.storage.tutti_store import stored_geometry

    s = stored_geometry(LLAMA3_8B, "fp8_block128")
    assert s["plane_bytes"] == LLAMA3_8B.plane_block_bytes * 33 // 64
    assert s["segment_bytes"] % 4096 == 0 and s["transform"] == 1
    m = stored_geometry(DEEPSEEK_V3_MLA, "fp8_block128")
    assert m["segment_bytes"] == 155648  # 4 x 38016 padded to 4 KiB
    assert stored_geometry(LLAMA3_8B)["segment_bytes"] == LLAMA3_8B.segment_bytes
    with pytest.raises(ValueError):
        stored_geometry(LLAMA3_8B, "int4")


def test_store_grows_segment_files_on_demand(tmp_path):
    """put_paged beyond the first file group materialises more groups instead of failing (posix, host pool)."""
    import numpy as np
    import torch

    from tutti_b200.index.chunk_index import chunk_keys_for_tokens
    from tutti_b200.models.kv_geometry import KVGeometry
    from tutti_b200.storage.tutti_store import TuttiKVStore

    g = KVGeometry("t-grow", num_layers=2, num_kv_heads=1, head_dim=128, chunk_tokens=64)
    st = TuttiKVStore(tmp_path, g, capacity_chunks=64, mounts=[str(tmp_path / "d0"), str(tmp_path / "d1")],
                      device=-1, backend="posix", segment_file_slots=4, runtime_options={"threads": 2})
    st.open()
    try:
        assert st.objects.ready_slots < 40
        pool = torch.randn(g.pool_shape(256), dtype=torch.bfloat16)
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(40 * 64)), 64, namespace=b"grow")
        src = np.arange(160).reshape(40, 4)
        st.put_paged(keys, src).wait()
        assert st.objects.ready_slots >= 40
        ref = pool[:, :, :160].clone()
        pool.zero_()
        st.get_paged(keys, src).wait()
        assert torch.equal(pool[:, :, :160], ref)
    finally:
        st.close()


def test_read_only_view_adopts_the_namespace_layout(tmp_path):
    """A view opened without the model's geometry lists exactly the committed chunks."""
    import numpy as np
    import torch

    from tutti_b200.index.chunk_index import chunk_keys_for_tokens
    from tutti_b200.models.kv_geometry import KVGeometry
    from tutti_b200.storage.object_layout import ObjectLayout
    from tutti_b200.storage.tutti_store import TuttiKVStore

    g = KVGeometry("t-view", num_layers=3, num_kv_heads=2, head_dim=128, chunk_tokens=64)
    mounts = [str(tmp_path / "d0"), str(tmp_path / "d1")]
    st = TuttiKVStore(tmp_path, g, capacity_chunks=64, mounts=mounts, device=-1, backend="posix",
                      segment_file_slots=4, runtime_options={"threads": 2})
    st.open()
    pool = torch.randn(g.pool_shape(64), dtype=torch.bfloat16)
    st.register_pool(pool)
    keys = chunk_keys_for_tokens(list(range(12 * 64)), 64, namespace=b"view")
    st.put_paged(keys, np.arange(48).reshape(12, 4)).wait()
    st.close()
    v = ObjectLayout.open_view(tmp_path, mounts)
    assert sorted(v.recover()) == sorted(keys)
    assert v.contains_prefix(keys, False) == 12
    v.close()
    with pytest.raises(Exception):
        ObjectLayout.open_view(tmp_path, mounts[:1])  # the namespace has two devices


def test_ready_markers_bind_segment_files_to_their_inode(tmp_path):
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    path = s.slot_path(0)
    marker = open(path + ".ready").read().split()
    st = os.stat(path)
    assert marker == ["tutti-ready", "v1", str(st.st_size), str(st.st_dev), str(st.st_ino)]
    assert os.path.exists(os.path.join(str(tmp_path / "d0"), ".tutti_segment_precreate.lock"))
    s.close()
    # a replacement file of the same name and size is not a prepared segment file
    data = open(path, "rb").read()
    with open(path + ".new", "wb") as f:  # created while the original exists: another inode
        f.write(data)
    os.replace(path + ".new", path)
    ro = core().ObjectStore()
    ro.open(cfg(tmp_path, read_only=True))
    assert ro.ready_slots == 0
    ro.close()
    # a writable open prepares that file again (new marker for the new inode)
    s = core().ObjectStore()
    s.open(cfg(tmp_path))
    assert s.ready_slots == 8
    assert open(path + ".ready").read().split()[4] == str(os.stat(path).st_ino)
    s.close()


def test_digests_match_tuttis_published_vectors():
    """CRC-32C and the object identity (FNV-1a + SplitMix64) against Tutti's digest contract values.

    Parity: reference tests/storage_objects/digest/object_digest_contract_test.cpp:80-101,180-189.
    """
    c = core()
    crc = {b"123456789": 0xE3069283, b"a": 0xC1D04330, b"abc": 0x364B3FB7, bytes(32): 0x8A9136AA,
           b"\xff" * 32: 0x62A8AB43, bytes(range(32)): 0x46DD794E}
    for data, want in crc.items():
        assert c.crc32c(data) == want, data
    ident = {b"": 0xF52A15E9A9B5E89B, b"abc": 0x0DD490490804B508, b"\xa1" * 16: 0x7ECB9653ACAF738B}
    for data, want in ident.items():
        assert c.object_identity(data) == want, data


def test_on_disk_structures_use_the_documented_offsets(tmp_path):
    """Object header, checkpoint container and residency bitmap: every fixed field at its documented offset.

    Parity: reference csrc/include/tutti/spi/storage_object_store.h:295-395 (the same offsets).
    """
    c = core()
    s = c.ObjectStore()
    s.open(cfg(tmp_path, rank_count=2))  # residency bitmaps exist when there are several ranks
    key = b"\x07" * 18
    (acc,), _ = s.reserve([key])
    s.commit([key])
    s.checkpoint()
    _, uri, off, slot, gen = acc
    with open(uri[len("file://"):], "rb") as f:
        f.seek(s.header_offset_for_slot(slot))
        h = f.read(4096)
    u32 = lambda b, o: struct.unpack_from("<I", b, o)[0]  # noqa: E731
    u64 = lambda b, o: struct.unpack_from("<Q", b, o)[0]  # noqa: E731
    assert h[:8] == b"TUTTIOBJ" and u32(h, 8) == 1 and u64(h, 16) == c.object_identity(key)
    assert u64(h, 24) == 3 * 8192 and u64(h, 32) == gen and u32(h, 40) == len(key)
    assert u32(h, 44) == c.crc32c(key) and u64(h, 48) > 0 and u32(h, 56) == c.crc32c(h[:56])
    assert h[64:64 + len(key)] == key and not any(h[64 + len(key):])  # key kept in the padding; rest zero
    ck = (tmp_path / "meta" / "checkpoint.bin").read_bytes()  # two mirrored containers, each a 4 KiB header + body
    live = [ck[i:i + 4096] for i in range(0, len(ck), 4096) if ck[i:i + 8] == b"TUTTIIDX"]
    assert live and all(u32(x, 8) == 1 for x in live)
    newest = max(live, key=lambda x: u64(x, 12))
    assert u64(newest, 20) > 0  # body bytes; the body's CRC sits at 28
    s.close()
    bm = next((tmp_path / "residency").glob("r0*"))
    b = bm.read_bytes()
    assert b[:8] == b"TUTTIRES" and u32(b, 8) == 1 and u32(b, 12) == 0 and u32(b, 16) == 2
    assert u64(b, 20) >= 16 and (b[4096 + slot // 8] >> (slot % 8)) & 1
