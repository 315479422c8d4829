"""The allocation-free C entry point ``tutti_nvme_io_noalloc``.

It serves callers that cannot allocate GPU memory while they move KV (engines
that hand all spare HBM to their KV pool at start-up, so a cudaMalloc mid-step
could fail; C-ABI embedders that own no CUDA allocator): its scratch lives in
a fixed device array inside the library. The test calls the exported C symbol through
ctypes and checks that two calls in a row restore exactly what the runtime's
ordinary submit path restores. The file is named to be collected last.
"""
import ctypes
import glob
import os

import numpy as np
import pytest
import torch

from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.models.kv_geometry import KVGeometry
from tutti_b200.storage.tutti_store import TuttiKVStore

pytestmark = pytest.mark.gpu

G = KVGeometry("noalloc-llama", num_layers=4, num_kv_heads=8, head_dim=128, chunk_tokens=64)


class Command(ctypes.Structure):
    _fields_ = [("logical", ctypes.c_uint64), ("target_row", ctypes.c_uint32), ("bytes", ctypes.c_uint32),
                ("first_piece", ctypes.c_uint32), ("n_pieces", ctypes.c_uint32), ("opcode", ctypes.c_uint16),
                ("transform", ctypes.c_uint16), ("replicas", ctypes.c_uint32)]


class Piece(ctypes.Structure):
    _fields_ = [("mem", ctypes.c_uint64), ("off", ctypes.c_uint32), ("bytes", ctypes.c_uint32)]


def _lib():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    path = glob.glob(os.path.join(root, "tutti_b200", "_core*.so"))[0]
    lib = ctypes.CDLL(path)
    lib.tutti_nvme_io_noalloc.restype = ctypes.c_int
    lib.tutti_nvme_io_noalloc.argtypes = [ctypes.c_void_p, ctypes.POINTER(Command), ctypes.c_uint32,
                                          ctypes.POINTER(Piece), ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32),
                                          ctypes.c_void_p]
    lib.tutti_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def build_commands(st, keys, dst_blocks, slot_bytes):
    """Coalesce the restore of ``keys`` into ``dst_blocks`` into commands of <= slot_bytes."""
    placements = []
    for k in keys:
        uri, off, _slot, _gen = st.objects.lookup(k)
        placements.append((uri[len("file://"):], off))
    tgts, toff, moff, lens = st.page_requests(placements, dst_blocks, np.arange(G.num_layers))
    rows = {int(h): st.runtime.target_row(int(h)) for h in np.unique(tgts)}
    base = st._pool[0].data_ptr()
    cmds, pieces = [], []
    for t, o, m, n in zip(tgts.tolist(), toff.tolist(), moff.tolist(), lens.tolist()):
        c = cmds[-1] if cmds else None
        if c is None or c.target_row != rows[t] or c.logical + c.bytes != o or c.bytes + n > slot_bytes:
            c = Command(logical=o, target_row=rows[t], bytes=0, first_piece=len(pieces), n_pieces=0, opcode=2)
            cmds.append(c)
        pieces.append(Piece(mem=base + m, off=c.bytes, bytes=n))
        c.bytes += n
        c.n_pieces += 1
    return (Command * len(cmds))(*cmds), len(cmds), (Piece * len(pieces))(*pieces), len(pieces)


def test_noalloc_entry_point_matches_runtime_submit_twice(tmp_path):
    slot = 1 << 20
    st = TuttiKVStore(tmp_path, G, capacity_chunks=32, mounts=[str(tmp_path / "nvme0")], device=0,
                      segment_file_slots=16,
                      runtime_options={"leases": 16, "max_ctas_per_op": 16, "slot_bytes": slot})
    st.open()
    try:
        nb = 256
        pool = torch.randn(G.pool_shape(nb), dtype=torch.bfloat16, device="cuda")
        st.register_pool(pool)
        n = 6
        keys = chunk_keys_for_tokens(list(range(n * 64)), 64, namespace=b"noalloc")
        rng = np.random.default_rng(3)
        blocks = rng.permutation(nb)
        src = blocks[: n * 4].reshape(n, 4)
        st.put_paged(keys, src).wait()
        # Existing entry point: the runtime's submit path.
        a = blocks[n * 4: n * 8].reshape(n, 4)
        st.get_paged(keys, a).wait()
        expect = pool[:, :, torch.from_numpy(a.reshape(-1)).cuda()].clone()
        lib = _lib()
        dp = st.runtime.gpu_path_address()
        stream = torch.cuda.current_stream()
        for call, region in enumerate((blocks[n * 8: n * 12], blocks[n * 12: n * 16])):
            dst = region.reshape(n, 4)
            idx = torch.from_numpy(dst.reshape(-1)).cuda()
            pool[:, :, idx] = 0
            torch.cuda.synchronize()
            cmds, nc, pcs, npc = build_commands(st, keys, dst, slot)
            status = (ctypes.c_uint32 * nc)()
            rc = lib.tutti_nvme_io_noalloc(ctypes.c_void_p(dp), cmds, nc, pcs, npc, status,
                                           ctypes.c_void_p(stream.cuda_stream))
            assert rc == 0, (call, rc, lib.tutti_noalloc_last_error())
            assert all(s == 0 for s in status)
            torch.cuda.synchronize()
            assert torch.equal(pool[:, :, idx], expect), f"call {call} differs from the runtime path"
        # Sizes beyond the fixed array are refused before launch.
        too_many = 4097
        big = (Command * too_many)()
        rc = lib.tutti_nvme_io_noalloc(ctypes.c_void_p(dp), big, too_many, pcs, npc, (ctypes.c_uint32 * too_many)(),
                                       ctypes.c_void_p(stream.cuda_stream))
        assert rc == -2 and b"MAX_COMMANDS" in lib.tutti_noalloc_last_error()
    finally:
        st.close()
