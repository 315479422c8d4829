"""GPU io kernel through the public API: emulated NVMe controllers, fused scatter/gather.

Failure cases are made on the host (the emulated controller completes with
an error status, or never posts a completion so the kernel's bounded wait
expires); nothing here faults or hangs the GPU.
"""
import os

import numpy as np
import pytest
import torch

from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.models.kv_geometry import KVGeometry
from tutti_b200.storage.base import StoreIOError
from tutti_b200.storage.tutti_store import TuttiKVStore

pytestmark = pytest.mark.gpu

G = KVGeometry("t-llama", num_layers=3, num_kv_heads=4, head_dim=128, chunk_tokens=64)


@pytest.fixture(params=["files", "memory"])
def media(request):
    """Emulated drive media: the backing files with page-locked host staging, or an
    in-memory image that the drives DMA from (copy engines) into HBM staging."""
    return request.param


def make(tmp_path, drives=1, media="files", **opts):
    base = {"leases": 8, "max_ctas_per_op": 8, "timeout_ms": 2000, "emulator_media": media}
    base.update(opts)
    st = TuttiKVStore(tmp_path, G, capacity_chunks=64, mounts=[str(tmp_path / f"nvme{d}") for d in range(drives)],
                      device=0, segment_file_slots=16, runtime_options=base)
    return st.open()


@pytest.mark.parametrize("drives", [1, 4])
def test_store_restore_roundtrip_random_blocks(tmp_path, drives, media):
    st = make(tmp_path, drives=drives, media=media)
    try:
        assert st.runtime.staging_on_device() == (media == "memory")
        nb = 512
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        n = 12
        keys = chunk_keys_for_tokens(list(range(n * 64)), 64, namespace=b"t")
        rng = np.random.default_rng(0)
        src = rng.permutation(nb)[: n * 4].reshape(n, 4)
        st.put_paged(keys, src).wait()
        ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
        dst = rng.permutation(nb)[: n * 4].reshape(n, 4)
        pool.zero_()
        st.get_paged(keys, dst).wait()
        got = pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()]
        assert torch.equal(got, ref)
        stats = st.runtime.controller_stats()
        assert sum(s["read_bytes"] for s in stats) == n * G.chunk_bytes
        if media == "memory":  # every command DMA'd by the copy engines, both directions
            assert sum(s["dma_copies"] for s in stats) >= n * G.chunk_bytes // (1 << 20)
    finally:
        st.close()


def test_restore_through_the_snvme_client_over_a_fake_driver(tmp_path, media):
    """The real-drive provider's path: the snvme client creates queue groups,
    maps rings and data buffers per page through the driver, has it create the
    queue pairs and hands the GPU data path BAR0 doorbells; a fake driver whose
    hardware is an emulated drive stands in for the kernel module."""
    st = make(tmp_path, drives=2, media=media, nvme_provider="snvme_fake", leases=40, max_ctas_per_op=16)
    try:
        stats = st.runtime.controller_stats()
        assert [s["kind"] for s in stats] == ["snvme", "snvme"]
        assert all(s["queues"] == 40 for s in stats)  # two queue groups (32 + 8) per drive
        nb = 512
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        n = 24
        keys = chunk_keys_for_tokens(list(range(n * 64)), 64, namespace=b"p1")
        rng = np.random.default_rng(3)
        src = rng.permutation(nb)[: n * 4].reshape(n, 4)
        st.put_paged(keys, src).wait()
        ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
        dst = rng.permutation(nb)[: n * 4].reshape(n, 4)
        pool.zero_()
        st.get_paged(keys, dst).wait()
        got = pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()]
        assert torch.equal(got, ref)
        stats = st.runtime.controller_stats()
        assert sum(s["read_bytes"] for s in stats) == n * G.chunk_bytes
    finally:
        st.close()


@pytest.mark.parametrize("provider", ["emulated", "snvme_fake"])
def test_direct_reads_land_in_the_pool_pages(tmp_path, provider):
    """With direct reads the drives DMA each read straight into the pool's
    pages (PRPs built by the io kernel from the pool's bus addresses): one
    copy per contiguous destination run instead of one per staged command."""
    copies = {}
    for direct in (False, True):
        root = tmp_path / f"d{int(direct)}"
        st = make(root, drives=2, media="memory", nvme_provider=provider, direct_reads=direct)
        try:
            nb = 512
            pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
            assert pool.data_ptr() % 4096 == 0
            st.register_pool(pool)
            n = 16
            keys = chunk_keys_for_tokens(list(range(n * 64)), 64, namespace=b"dr")
            rng = np.random.default_rng(7)
            src = rng.permutation(nb)[: n * 4].reshape(n, 4)
            st.put_paged(keys, src).wait()
            ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
            before = sum(s["dma_copies"] for s in st.runtime.controller_stats())
            dst = rng.permutation(nb)[: n * 4].reshape(n, 4)
            pool.zero_()
            st.get_paged(keys, dst).wait()
            assert torch.equal(pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()], ref)
            # a layer subset goes the same way
            pool.zero_()
            st.get_paged(keys, dst, layers=[1]).wait()
            got = pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()]
            assert torch.equal(got[1], ref[1]) and torch.count_nonzero(got[0]) == 0
            copies[direct] = sum(s["dma_copies"] for s in st.runtime.controller_stats()) - before
        finally:
            st.close()
    # staged: about one copy per command; direct: one per destination block plane
    assert copies[True] > 2 * copies[False]


def test_layer_subset_restore(tmp_path, media):
    st = make(tmp_path, media=media)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64)
        src = np.arange(8).reshape(2, 4)
        st.put_paged(keys, src).wait()
        ref = pool.clone()
        dst = (np.arange(8) + 16).reshape(2, 4)
        pool[:, :, 16:24].zero_()
        st.get_paged(keys, dst, layers=[1]).wait()
        assert torch.equal(pool[1, :, 16:24], ref[1, :, 0:8])
        assert torch.count_nonzero(pool[0, :, 16:24]) == 0
        assert torch.count_nonzero(pool[2, :, 16:24]) == 0
    finally:
        st.close()


def test_media_error_reports_failed_requests(tmp_path, media):
    st = make(tmp_path, media=media)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64)
        st.put_paged(keys, np.arange(8).reshape(2, 4)).wait()
        st.runtime.inject(0, "media_error", 1)
        with pytest.raises(StoreIOError) as ei:
            st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4)).wait()
        assert "nvme_cq_error" in ei.value.kind
        assert len(ei.value.failed) > 0
        # the path keeps working after the error
        st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4)).wait()
    finally:
        st.close()


def test_lost_completion_times_out_and_queue_recovers(tmp_path, media):
    st = make(tmp_path, timeout_ms=500, media=media)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64)
        st.put_paged(keys, np.arange(8).reshape(2, 4)).wait()
        ref = pool[:, :, 0:8].clone()
        st.runtime.inject(0, "drop_completion", 1)
        with pytest.raises(StoreIOError) as ei:
            st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4)).wait()
        assert "cq_timeout" in ei.value.kind
        # queues were reset after the timeout: a fresh restore is exact
        st.get_paged(keys, (np.arange(8) + 16).reshape(2, 4)).wait()
        assert torch.equal(pool[:, :, 16:24], ref)
    finally:
        st.close()


def test_enqueue_wait_orders_consumer_stream(tmp_path, media):
    st = make(tmp_path, media=media)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(64)), 64)
        st.put_paged(keys, np.arange(4).reshape(1, 4)).wait()
        ref = pool[:, :, 0:4].clone()
        io_stream = torch.cuda.Stream()
        comp = st.get_paged(keys, np.arange(4).reshape(1, 4) + 8, stream=io_stream)
        consumer = torch.cuda.Stream()
        comp.enqueue_wait(consumer)
        with torch.cuda.stream(consumer):
            out = pool[:, :, 8:12].clone()
        consumer.synchronize()
        comp.wait()
        assert torch.equal(out, ref)
    finally:
        st.close()


def _fp8_roundtrip_pages(pages: torch.Tensor) -> torch.Tensor:
    """Standalone block-scaling kernels on whole pages: the bytes the fused path must reproduce."""
    from tutti_b200 import ops

    rows = pages.reshape(-1, pages[0, 0, 0].numel())
    q, s = ops.fp8_quant(rows)
    return ops.fp8_dequant(q, s).reshape(pages.shape)


@pytest.mark.parametrize("drives", [1, 3])
def test_fp8_stored_format_quantises_on_store_and_dequantises_on_restore(tmp_path, drives, media):
    st = TuttiKVStore(tmp_path, G, capacity_chunks=64, mounts=[str(tmp_path / f"nvme{d}") for d in range(drives)],
                      device=0, segment_file_slots=16, stored_format="fp8_block128",
                      runtime_options={"leases": 8, "max_ctas_per_op": 8, "timeout_ms": 2000,
                                       "emulator_media": media})
    st.open()
    try:
        nb = 256
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda") * 3
        pool[:, :, 5].zero_()  # an all-zero page: scale 1, zeros back
        st.register_pool(pool)
        n = 10
        keys = chunk_keys_for_tokens(list(range(n * 64)), 64, namespace=b"f8")
        rng = np.random.default_rng(1)
        src = rng.permutation(nb)[: n * 4].reshape(n, 4)
        src[0, 0] = 5
        st.put_paged(keys, src).wait()
        sidx = torch.from_numpy(src.reshape(-1)).cuda()
        orig = pool[:, :, sidx].clone()
        want = _fp8_roundtrip_pages(orig)
        # stored bytes are 33/64 of the pool bytes
        stats = st.runtime.controller_stats()
        assert sum(x["write_bytes"] for x in stats) == n * G.num_layers * 4 * G.planes * st.stored["plane_bytes"]
        dst = rng.permutation(nb)[: n * 4].reshape(n, 4)
        pool.zero_()
        st.get_paged(keys, dst).wait()
        got = pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()]
        assert torch.equal(got, want)  # identical to the standalone kernels
        # and within E4M3 precision of the fp32 source: |err| <= amax(group) / 16
        ref = orig.float().reshape(-1, 128)
        amax = ref.abs().amax(dim=1, keepdim=True)
        assert torch.all((got.float().reshape(-1, 128) - ref).abs() <= amax / 16 + 1e-6)
        # layer subset restore of the transformed format
        pool.zero_()
        st.get_paged(keys[:2], dst[:2], layers=[1]).wait()
        d2 = torch.from_numpy(dst[:2].reshape(-1)).cuda()
        assert torch.equal(pool[1, :, d2], want[1, :, :8])
        assert torch.count_nonzero(pool[0]) == 0
    finally:
        st.close()


def test_subsector_index_pages_pack_into_aligned_commands(tmp_path, media):
    # DeepSeek-V3.2-style index cache: 132 bytes per token, 8,448-byte pages (not a sector multiple)
    gi = KVGeometry("t-idx", num_layers=3, num_kv_heads=1, head_dim=132, block_size=64, planes=1,
                    dtype=torch.uint8, chunk_tokens=256)
    st = TuttiKVStore(tmp_path, gi, capacity_chunks=32, mounts=[str(tmp_path / f"nvme{d}") for d in range(2)],
                      device=0, segment_file_slots=16,
                      runtime_options={"leases": 8, "max_ctas_per_op": 8, "emulator_media": media})
    st.open()
    try:
        nb = 64
        pool = torch.randint(0, 256, gi.pool_shape(nb), dtype=torch.uint8, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(5 * 256)), 256, namespace=b"idx")
        rng = np.random.default_rng(2)
        src = rng.permutation(nb)[:20].reshape(5, 4)
        st.put_paged(keys, src).wait()
        ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
        dst = rng.permutation(nb)[:20].reshape(5, 4)
        pool.zero_()
        st.get_paged(keys, dst).wait()
        assert torch.equal(pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()], ref)
    finally:
        st.close()


@pytest.mark.parametrize("consumer_drain", [False, True])
def test_split_completion_restores_exactly(tmp_path, consumer_drain, media):
    # submit-phase launch queues the reads and exits; the drain runs on the
    # consumer stream (enqueue_wait) or, without one, from the host fallback
    st = make(tmp_path, drives=2, async_completion=True, slots_per_lease=8, media=media)
    try:
        nb = 256
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(10 * 64)), 64, namespace=b"split")
        rng = np.random.default_rng(4)
        src = rng.permutation(nb)[:40].reshape(10, 4)
        st.put_paged(keys, src).wait()
        ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
        for it in range(2):
            dst = rng.permutation(nb)[:40].reshape(10, 4)
            pool.zero_()
            io_stream = torch.cuda.Stream()
            comp = st.get_paged(keys, dst, stream=io_stream)
            didx = torch.from_numpy(dst.reshape(-1)).cuda()
            if consumer_drain:
                consumer = torch.cuda.Stream()
                comp.enqueue_wait(consumer)
                with torch.cuda.stream(consumer):
                    out = pool[:, :, didx].clone()
                consumer.synchronize()
                comp.wait()
            else:
                comp.wait()
                out = pool[:, :, didx]
            assert torch.equal(out, ref), it
    finally:
        st.close()


def test_split_completion_deadline_runs_from_submission(tmp_path, media):
    st = make(tmp_path, async_completion=True, timeout_ms=500, media=media)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64)
        st.put_paged(keys, np.arange(8).reshape(2, 4)).wait()
        ref = pool[:, :, 0:8].clone()
        st.runtime.inject(0, "drop_completion", 1)
        with pytest.raises(StoreIOError) as ei:
            st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4)).wait()
        assert "cq_timeout" in ei.value.kind
        st.get_paged(keys, (np.arange(8) + 16).reshape(2, 4)).wait()
        assert torch.equal(pool[:, :, 16:24], ref)
    finally:
        st.close()


def test_restore_on_a_green_context_io_stream(tmp_path):
    # io kernels on a stream confined to a 16-SM partition of the GPU
    from tutti_b200.parallel.green_context import GreenIoStream

    g = GreenIoStream(16, 0)
    st = make(tmp_path, max_ctas_per_op=8)
    try:
        assert 16 <= g.sms < torch.cuda.get_device_properties(0).multi_processor_count
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(4 * 64)), 64, namespace=b"green")
        st.put_paged(keys, np.arange(16).reshape(4, 4)).wait()
        ref = pool[:, :, 0:16].clone()
        comp = st.get_paged(keys, (np.arange(16) + 32).reshape(4, 4), stream=g.stream)
        comp.wait()
        g.stream.synchronize()
        assert torch.equal(pool[:, :, 32:48], ref)
    finally:
        st.close()
        g.close()


def test_data_path_host_fault_seams(tmp_path):
    """Launch failure: nothing issued, all rejected; event-record failure: settled from statuses; query error: FAILED."""
    st = make(tmp_path, max_ctas_per_op=2)  # the op failed by a query error keeps its (at most 2) leases
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64, namespace=b"seams")
        st.put_paged(keys, np.arange(8).reshape(2, 4)).wait()
        ref = pool[:, :, 0:8].clone()
        free = st.runtime.free_leases()

        st.runtime.testing_inject_data_path("launch_failure", 1)
        with pytest.raises(StoreIOError) as ei:
            st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4)).wait()
        assert ei.value.kind == "rejected" and "injected" in str(ei.value)
        assert st.runtime.free_leases() == free  # nothing was issued, every lease came back

        pool[:, :, 16:24].zero_()
        st.runtime.testing_inject_data_path("event_record_failure", 1)
        st.get_paged(keys, (np.arange(8) + 16).reshape(2, 4)).wait()  # the IO ran: settled synchronously
        assert torch.equal(pool[:, :, 16:24], ref)

        st.runtime.testing_inject_data_path("query_error", 1)
        with pytest.raises(StoreIOError):
            st.get_paged(keys, (np.arange(8) + 24).reshape(2, 4)).wait()
        # the path still serves restores (the failed op keeps its leases: its device state is unknown)
        pool[:, :, 32:40].zero_()
        st.get_paged(keys, (np.arange(8) + 32).reshape(2, 4)).wait()
        assert torch.equal(pool[:, :, 32:40], ref)
    finally:
        st.close()


def test_event_record_failure_on_a_split_read_settles_after_the_drain(tmp_path):
    st = make(tmp_path, async_completion=True)
    try:
        nb = 64
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(2 * 64)), 64, namespace=b"seams2")
        st.put_paged(keys, np.arange(8).reshape(2, 4)).wait()
        ref = pool[:, :, 0:8].clone()
        pool[:, :, 8:16].zero_()
        st.runtime.testing_inject_data_path("event_record_failure", 1)
        comp = st.get_paged(keys, (np.arange(8) + 8).reshape(2, 4))
        consumer = torch.cuda.Stream()
        comp.enqueue_wait(consumer)  # a settled op needs no drain: nothing is launched
        comp.wait()
        assert torch.equal(pool[:, :, 8:16], ref)
    finally:
        st.close()


def test_split_completion_of_an_op_larger_than_its_leased_slots(tmp_path, media):
    # 2 CTAs x 2 slots hold 4 commands; the op has 12: the drain takes over the
    # submitted ones and claims the rest itself
    st = make(tmp_path, drives=2, async_completion=True, max_ctas_per_op=2, slots_per_lease=2, media=media)
    try:
        nb = 256
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(12 * 64)), 64, namespace=b"split-big")
        rng = np.random.default_rng(5)
        src = rng.permutation(nb)[:48].reshape(12, 4)
        st.put_paged(keys, src).wait()
        ref = pool[:, :, torch.from_numpy(src.reshape(-1)).cuda()].clone()
        dst = rng.permutation(nb)[:48].reshape(12, 4)
        pool.zero_()
        comp = st.get_paged(keys, dst, stream=torch.cuda.Stream())
        assert st.runtime.last_submit_profile()["commands"] > 4
        consumer = torch.cuda.Stream()
        comp.enqueue_wait(consumer)
        with torch.cuda.stream(consumer):
            out = pool[:, :, torch.from_numpy(dst.reshape(-1)).cuda()].clone()
        consumer.synchronize()
        comp.wait()
        assert torch.equal(out, ref)
    finally:
        st.close()
