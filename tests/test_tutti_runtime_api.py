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


def test_factories_take_tutti_presets(tmp_path):
    stub = tutti_runtime.make_stub_runtime()
    assert isinstance(stub, tutti_runtime.Runtime)
    with pytest.raises(ValueError, match="raid0"):
        tutti_runtime.make_raid0_nvme_runtime({"devices": [{"mount_path": str(tmp_path / "a")}]})
