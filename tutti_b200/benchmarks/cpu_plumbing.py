"""CPU plumbing: StorageRuntime over the POSIX backend with a Llama-3-8B-shaped paged KV pool.

    python -m tutti_b200.benchmarks.cpu_plumbing [--blocks 1000] [--seed 0] [--drives 2]

No GPU and no NVMe. The pool is ``[32 layers, K/V, blocks, 16 tokens, 8 KV
heads, 128]`` bf16 values ~ N(0, 1) from ``--seed`` (64 KiB of K+V per block
per layer). The blocks sit at a seeded random permutation of the pool's slots
and are written, in that order, as chunks of 8 blocks (128 tokens) through
``TuttiKVStore.put_paged`` (host-executed pwrite). They are read back through
``get_paged`` into a second pool at a different permutation, then checked:

* every block's bytes equal the written block's;
* every chunk's object sits where the segment-file format puts it: path
  ``<mount[slot % N]>/r0/segments/<(slot / N) / slots_per_file>.seg``, object
  header (``TUTTIOBJ``, payload bytes, the key) at the slot's region, and its
  payload, read with plain file IO, is the chunk's layers in order, each
  layer the chunk's blocks with K then V.

Prints one JSON line (write and read GB/s, checks).
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import struct
import tempfile
import time

import numpy as np
import torch

BLOCKS_PER_CHUNK = 8


def run(blocks: int = 1000, seed: int = 0, drives: int = 2, root: str | None = None) -> dict:
    from ..index.chunk_index import chunk_keys_for_tokens
    from ..models.kv_geometry import KVGeometry
    from ..storage.tutti_store import TuttiKVStore

    if blocks % BLOCKS_PER_CHUNK:
        raise ValueError(f"blocks must be a multiple of {BLOCKS_PER_CHUNK}")
    g = KVGeometry("llama-3-8b", num_layers=32, num_kv_heads=8, head_dim=128, block_size=16,
                   chunk_tokens=16 * BLOCKS_PER_CHUNK)
    chunks = blocks // BLOCKS_PER_CHUNK
    own = root is None
    root = root or tempfile.mkdtemp(prefix="tutti_plumb_")
    out = {"bench": "cpu_plumbing", "blocks": blocks, "chunks": chunks, "layers": g.num_layers,
           "block_layer_bytes": g.block_layer_bytes, "seed": seed}
    t_start = time.perf_counter()
    try:
        pool_a = torch.empty(g.pool_shape(blocks), dtype=torch.bfloat16)
        rng = np.random.default_rng(seed)
        for layer in range(g.num_layers):  # one layer of fp32 at a time: no pool-sized temporary
            vals = rng.standard_normal(pool_a[layer].numel(), dtype=np.float32)
            pool_a[layer] = torch.from_numpy(vals).view(pool_a[layer].shape).to(torch.bfloat16)
        pool_b = torch.zeros_like(pool_a)
        t_gen = time.perf_counter()
        src = np.random.default_rng(seed).permutation(blocks).reshape(chunks, BLOCKS_PER_CHUNK)
        dst = np.random.default_rng(seed + 1).permutation(blocks).reshape(chunks, BLOCKS_PER_CHUNK)
        keys = chunk_keys_for_tokens(list(range(blocks * 16)), g.chunk_tokens, namespace=b"plumbing")
        mounts = [os.path.join(root, f"disk{d}") for d in range(drives)]
        st = TuttiKVStore(root, g, capacity_chunks=chunks, mounts=mounts, backend="posix", device=-1,
                          segment_file_slots=16, runtime_options={"threads": 8, "direct_io": True})
        st.open()
        try:
            st.layout.precreate_until(chunks)
            nbytes = blocks * g.num_layers * g.block_layer_bytes
            st.register_pool(pool_a)
            t0 = time.perf_counter()
            st.put_paged(keys, src).wait()
            t1 = time.perf_counter()
            st.register_pool(pool_b)
            t2 = time.perf_counter()
            st.get_paged(keys, dst).wait()
            t3 = time.perf_counter()
            out["write_GBps"] = round(nbytes / (t1 - t0) / 1e9, 3)
            out["read_GBps"] = round(nbytes / (t3 - t2) / 1e9, 3)
            out["bytes"] = nbytes
            out["blocks_equal"] = all(  # chunk by chunk: no pool-sized temporaries
                torch.equal(pool_b[:, :, torch.from_numpy(dst[i])], pool_a[:, :, torch.from_numpy(src[i])])
                for i in range(chunks))
            t4 = time.perf_counter()
            out["layout_ok"], out["layout_detail"] = check_layout(st, g, keys, pool_a, src, mounts)
            out["phase_s"] = {"fill_pools": round(t_gen - t_start, 1), "open_precreate": round(t0 - t_gen, 1),
                              "write": round(t1 - t0, 2), "read": round(t3 - t2, 2), "verify_blocks": round(t4 - t3, 1),
                              "verify_layout": round(time.perf_counter() - t4, 1)}
        finally:
            st.close()
    finally:
        if own:
            shutil.rmtree(root, ignore_errors=True)
    out["ok"] = out.get("blocks_equal", False) and out.get("layout_ok", False)
    return out


def check_layout(st, g, keys, pool, src, mounts) -> tuple[bool, str]:
    """Re-read every chunk with plain file IO and compare with the segment-file format."""
    objs = st.objects
    n = len(mounts)
    seg = st.stored["segment_bytes"]
    files = set()
    for i, key in enumerate(keys):
        uri, payload_off, slot, _gen = objs.lookup(bytes(key))
        path = uri[len("file://"):]
        want = os.path.join(mounts[slot % n], "r0", "segments", f"{(slot // n) // st.layout.segment_file_slots}.seg")
        if os.path.normpath(path) != os.path.normpath(want):
            return False, f"chunk {i}: slot {slot} at {path}, expected {want}"
        hdr_off = objs.header_offset_for_slot(slot)
        if payload_off != hdr_off + st.layout.segment_header_bytes:
            return False, f"chunk {i}: payload offset {payload_off} != header {hdr_off} + prefix"
        with open(path, "rb") as f:
            f.seek(hdr_off)
            hdr = f.read(64 + len(key))
            f.seek(payload_off)
            payload = f.read(g.num_layers * seg)
        if hdr[:8] != b"TUTTIOBJ":
            return False, f"chunk {i}: bad header magic {hdr[:8]!r}"
        payload_bytes, = struct.unpack_from("<Q", hdr, 24)
        key_len, = struct.unpack_from("<I", hdr, 40)
        if payload_bytes != g.num_layers * seg or hdr[64:64 + key_len] != bytes(key):
            return False, f"chunk {i}: header fields do not match"
        # expected payload: per layer, the chunk's blocks in order, each K then V, padded to the segment
        blk = pool[:, :, torch.from_numpy(src[i])]                     # [L, P, b, ...]
        body = blk.permute(0, 2, 1, 3, 4, 5).contiguous().view(torch.uint8).reshape(g.num_layers, -1)
        got = torch.frombuffer(bytearray(payload), dtype=torch.uint8).reshape(g.num_layers, seg)
        if not torch.equal(got[:, :body.shape[1]], body):
            return False, f"chunk {i}: payload bytes differ from the pool's blocks"
        files.add(path)
    return True, f"{len(keys)} chunks in {len(files)} segment files"


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--blocks", type=int, default=1000)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--drives", type=int, default=2)
    a = p.parse_args(argv)
    r = run(a.blocks, a.seed, a.drives)
    print(json.dumps(r))
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
