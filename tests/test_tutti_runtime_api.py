"""``tutti_runtime``: Tutti's binding surface (6-tuple submits, wait results) over this build's runtime."""
import numpy as np
import pytest

import tutti_runtime
from tutti_b200._native import core


def memfs_runtime():
    return tutti_runtime.Runtime(core().make_memfs_runtime(capacity_bytes=1 << 20))


def test_mixed_submit_wait_and_retained_results():
    rt = memfs_runtime()
    t = rt.open_batch(["memfs://obj?size=64K"])[0]
    src = np.arange(8192, dtype=np.uint8)
    dst = np.zeros(8192, dtype=np.uint8)
    ms = rt.register_memory(src.ctypes.data, src.nbytes, "HOST")
    md = rt.register_memory(dst.ctypes.data, dst.nbytes, "host")
    w = rt.submit([(t, 0, ms, 0, 4096, "write"), (t, 65536, ms, 0, 4096, "write")], accel_id=0, stream=None,
                  execution="host")
    assert w.io_handle is not None and w.rejected == [1] and w.initial_states == [True, False]
    assert rt.wait(w.io_handle, 1000) == ("OK", "COMPLETED")
    rt.release_io(w.io_handle)
    assert rt.query_io(w.io_handle) == "COMPLETED" and rt.wait_result(w.io_handle).confirmed_bytes == 4096
    # one submit mixing a read of what was written and another write
    m = rt.submit([(t, 0, md, 0, 4096, "read"), (t, 8192, ms, 4096, 4096, "write")], 0, None, "host")
    assert m.status_ok and m.rejected == [] and rt.open_io_count() == 1
    d = rt.wait_detail(m.io_handle, 1000)
    assert d["state"] == "COMPLETED" and d["confirmed_bytes"] == 8192 and d["failure_scope"] == "NONE"
    rt.release_io(m.io_handle)
    assert np.array_equal(dst[:4096], src[:4096]) and rt.open_io_count() == 0
    with pytest.raises(ValueError):
        rt.submit([(t, 0, md, 0, 4096, "read")], 0, None, "device")  # device execution needs a stream
    with pytest.raises(ValueError):
        rt.submit([(t, 0, md, 0, 4096)], 0, None, "host")
    rt.shutdown(1000)


def test_stub_runtime_ios_stay_in_flight_until_forced():
    import numpy as np

    rt = tutti_runtime.make_stub_runtime()
    buf = np.zeros(8192, dtype=np.uint8)
    mem = rt.register_memory(buf.ctypes.data, buf.nbytes, "host")
    (t,) = rt.open_batch(["file:///no/such/file"])  # any URI: a stub target
    r = rt.submit([(t, 0, mem, 0, 4096, "read"), (t, 4096, mem, 4096, 8192, "write")], -1, None, "host")
    assert r.initial_states == [True, False] and r.io_handle is not None  # the second overruns the memory
    assert rt.query_io(r.io_handle) == "IN_FLIGHT" and rt.wait(r.io_handle, 5) == ("TIMEOUT", "IN_FLIGHT")
    rt.testing_force_complete(r.io_handle, "FAILED")
    res = rt.wait_result(r.io_handle, 0)
    assert res.state == "FAILED" and res.failed_request_indices == [0]
    rt.release_io(r.io_handle)
    assert rt.query_io(r.io_handle) == "FAILED"  # retained after release
    r2 = rt.submit([(t, 0, mem, 0, 4096, "write")], -1, None, "host")
    with pytest.raises(ValueError):
        rt.testing_force_complete(r2.io_handle, "DONE")
    rt.testing_force_complete(r2.io_handle, "COMPLETED")
    assert rt.wait(r2.io_handle, 0) == ("OK", "COMPLETED")
    rt.release_io(r2.io_handle)
    assert rt.open_io_count() == 0
    rt.shutdown(100)


def test_force_complete_is_refused_on_a_component_backed_runtime(tmp_path):
    import numpy as np

    from tutti_b200._native import core

    native = core().make_posix_runtime(-1, [str(tmp_path)])
    rt = tutti_runtime.Runtime(native)
    p = tmp_path / "f.bin"
    p.write_bytes(b"x" * 8192)
    (t,) = rt.open_batch([f"file://{p}"])
    buf = np.zeros(4096, dtype=np.uint8)
    mem = rt.register_memory(buf.ctypes.data, buf.nbytes, "host")
    r = rt.submit([(t, 0, mem, 0, 4096, "read")], -1, None, "host")
    rt.wait(r.io_handle, 5000)
    with pytest.raises(Exception, match="stub"):
        rt.testing_force_complete(r.io_handle, "COMPLETED")
    rt.release_io(r.io_handle)
    rt.shutdown(1000)


def test_factories_take_tutti_presets(tmp_path):
    stub = tutti_runtime.make_stub_runtime()
    assert isinstance(stub, tutti_runtime.Runtime)
    with pytest.raises(ValueError, match="raid0"):
        tutti_runtime.make_raid0_nvme_runtime({"devices": [{"mount_path": str(tmp_path / "a")}]})


def test_object_store_with_tutti_config(tmp_path):
    s = tutti_runtime.ObjectStore()
    cfg = {"uri": str(tmp_path), "devices": [{"mount_path": str(tmp_path / "d0"), "namespace_id": 1},
                                             {"mount_path": str(tmp_path / "d1")}],
           "segment_bytes": 8192, "segment_count": 2, "segment_file_slots": 4, "segment_header_bytes": 131072,
           "capacity_slots": 16, "namespace_fingerprint": b"\x01geometry", "rank_id": 0, "rank_count": 1,
           "background_reclaim": True, "residency_sync_interval_ms": 100}
    with pytest.raises(ValueError):
        s.open("local_nvme_file", cfg)  # one device only
    s.open("striped_local_nvme_file", cfg)
    assert s.is_open() and s.ready_slots() == 8
    keys = [bytes([i]) * 18 for i in range(3)]
    acc, rej = s.reserve(keys)
    s.commit([a[0] for a in acc])
    assert s.contains_prefix(keys) == 3 and s.contains_prefix_all_ranks(keys) == 3
    s.close()
    again = tutti_runtime.ObjectStore()
    with pytest.raises(Exception):  # another geometry fingerprint fails closed
        again.open("striped_local_nvme_file", dict(cfg, namespace_fingerprint=b"other"))
    again = tutti_runtime.ObjectStore()
    again.open("striped_local_nvme_file", cfg)
    assert sorted(again.recover()) == sorted(keys)
    again.close()


def test_memory_store_with_tutti_names_and_host_buffers():
    from tutti.storage.memory import MemoryKVStore

    s = MemoryKVStore(segment_bytes=4096, num_chunks=4)
    s.open()
    src, dst = bytearray(range(256)) * 16, bytearray(4096)
    a, b = s.register_buffer(src, 4096), s.register_buffer(memoryview(dst), 4096)
    s.put_batch([(b"k" * 18, a, 0)]).wait()
    s.get_batch([(b"k" * 18, b, 0)]).wait()
    assert dst == src
    with pytest.raises(ValueError):
        MemoryKVStore(num_chunks=4)


def test_error_injection_hook_needs_emulated_drives():
    rt = memfs_runtime()
    with pytest.raises((IndexError, ValueError)):
        rt.testing_inject_next_read_nvme_error(0x285)
    rt.shutdown(1000)
