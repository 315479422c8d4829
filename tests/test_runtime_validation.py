"""Runtime-level validation of transformed and sub-sector requests (host only, posix data path)."""
import numpy as np
import pytest
import torch

from tutti_b200._native import core


@pytest.fixture
def rt(tmp_path):
    (tmp_path / "d0").mkdir()
    f = tmp_path / "d0" / "seg.bin"
    f.write_bytes(b"\0" * (1 << 20))
    r = core().make_posix_runtime(-1, [str(tmp_path / "d0")], {"threads": 1})
    h = r.open("file://" + str(f))
    yield r, h
    r.shutdown(10_000)


def _submit(r, h, mem, transform, plane=1024, planes=1, blocks=4):
    geo = {"planes": planes, "plane_bytes": plane, "segment_bytes": 65536, "block_layer_bytes": plane * planes,
           "num_blocks": 16, "transform": transform}
    return r.submit_paged("read", mem, np.asarray([h], np.uint64), np.asarray([0], np.uint64),
                          np.arange(blocks, dtype=np.int64).reshape(1, blocks), np.arange(1, dtype=np.int64), geo, 0,
                          True)


def test_fp8_transform_rejected_by_a_data_path_without_it(rt):
    r, h = rt
    buf = torch.zeros(1 << 16, dtype=torch.uint8)
    mem = r.register_memory(buf.data_ptr(), buf.numel(), "host", -1)
    out = _submit(r, h, mem, transform=1)
    assert len(out["rejected"]) == 4 and "fp8 block transform" in " ".join(out["reasons"])
    ok = _submit(r, h, mem, transform=0)
    assert not ok["rejected"]
    r.wait(ok["io"], 10_000)
    r.release_io(ok["io"])


def test_unknown_transform_rejected(rt):
    r, h = rt
    buf = torch.zeros(1 << 16, dtype=torch.uint8)
    mem = r.register_memory(buf.data_ptr(), buf.numel(), "host", -1)
    with pytest.raises(ValueError):
        _submit(r, h, mem, transform=7)
