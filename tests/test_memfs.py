"""memfs sample backend: a resolver, payload, DataPath and byte budget written only against the SPI.

Parity: reference csrc/payloads/memfs (sample DataPath) and csrc/resource/memory.
"""
import numpy as np
import pytest

from tutti_b200._native import core


def A(*x):
    return np.array(x, dtype=np.uint64)


def make(cap=1 << 20):
    return core().make_memfs_runtime(capacity_bytes=cap)


def test_write_then_read_back_host_memory():
    rt = make()
    t = rt.open("memfs://kv0?size=256K")
    assert rt.query_target(t)["data_path"] == "memfs"
    src = np.random.default_rng(0).integers(0, 256, 65536, dtype=np.uint8)
    dst = np.zeros(2 * 65536, dtype=np.uint8)
    ms = rt.register_memory(src.ctypes.data, src.nbytes, "host")
    md = rt.register_memory(dst.ctypes.data, dst.nbytes, "host")
    w = rt.submit_arrays("write", A(ms), A(0), A(t), A(4096), A(65536), 0, True)
    assert w["ok"]
    assert rt.wait(w["io"])["state"] == "completed"
    rt.release_io(w["io"])
    # two reads: the written range and an untouched (zero) range
    r = rt.submit_arrays("read", A(md), A(0, 65536), A(t), A(4096, 131072), A(65536, 65536), 0, True)
    res = rt.wait(r["io"])
    assert res["state"] == "completed" and res["confirmed_bytes"] == 2 * 65536
    rt.release_io(r["io"])
    assert np.array_equal(dst[:65536], src)
    assert not dst[65536:].any()


def test_requests_outside_the_object_are_rejected_individually():
    rt = make()
    t = rt.open("memfs://small?size=4K")
    buf = np.zeros(8192, dtype=np.uint8)
    m = rt.register_memory(buf.ctypes.data, buf.nbytes, "host")
    r = rt.submit_arrays("read", A(m), A(0, 0), A(t), A(0, 2048), A(4096, 4096), 0, True)
    assert r["rejected"] == [1]  # partial commit: the in-range request ran
    assert rt.wait(r["io"])["confirmed_bytes"] == 4096
    rt.release_io(r["io"])


def test_budget_and_namespace():
    rt = make(cap=1 << 20)
    a = rt.open("memfs://a?size=768K")
    with pytest.raises(Exception, match="budget"):
        rt.open("memfs://b?size=512K")  # over the 1 MiB budget
    assert rt.memfs_usage()["used"] == 768 << 10
    a2 = rt.open("memfs://a")  # an existing object by name
    assert rt.query_target(a2)["size"] == 768 << 10
    with pytest.raises(Exception, match="another size"):
        rt.open("memfs://a?size=4K")
    with pytest.raises(Exception, match="no memfs object"):
        rt.open("memfs://missing")
    rt.memfs_remove("a")
    assert rt.memfs_usage()["used"] == 768 << 10  # open targets keep the bytes
    rt.close(a)
    rt.close(a2)
    assert rt.memfs_usage()["used"] == 0
    rt.open("memfs://b?size=512K")


@pytest.mark.gpu
def test_device_memory_roundtrip():
    import torch

    rt = make()
    t = rt.open("memfs://dev?size=1M")
    x = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device="cuda")
    y = torch.zeros_like(x)
    mx = rt.register_memory(x.data_ptr(), x.numel(), "device", 0)
    my = rt.register_memory(y.data_ptr(), y.numel(), "device", 0)
    torch.cuda.synchronize()
    w = rt.submit_arrays("write", A(mx), A(0), A(t), A(0), A(1 << 20), 0, True)
    rt.wait(w["io"])
    rt.release_io(w["io"])
    r = rt.submit_arrays("read", A(my), A(0), A(t), A(0), A(1 << 20), 0, True)
    assert rt.wait(r["io"])["state"] == "completed"
    rt.release_io(r["io"])
    assert torch.equal(x, y)
