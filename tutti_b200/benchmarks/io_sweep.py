"""Single-GPU restore bandwidth against batch size and against io-kernel width.

    python -m tutti_b200.benchmarks.io_sweep [--drives 4] [--iters 5] [--warmup 3]

The unit is a 64 KiB page: one (block, layer) of Llama-3.1-8B's KV (16 tokens
× 8 KV heads × 128 × bf16 × K and V). A restore of ``chunks`` chunks and ``L``
layers reads ``chunks × 16 × L`` pages through the public ``get_paged`` path
(emulated NVMe controllers over page-cached files, fused scatter into the
paged pool). Two sweeps, as the reference tabulates them:

* ``batch``: pages per restore ≈ 128, 486, 972, 1944, 3888 at the default width;
* ``width``: ≈ 486 pages per restore with ``max_ctas_per_op`` (queue leases,
  one CTA each, ``slots_per_lease`` commands in flight per CTA) swept; the
  reference sweeps its submit kernel's worker-thread pool instead.

Time is CUDA-event time around ``get_paged(...).wait()`` after warm-up,
including the host side of the emulated drives. Prints one JSON line.
Parity: reference doc/design/kv-storage-layout-and-io-submission.md:168-170
(read vs workers) and :273-275 (read vs batch size).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import tempfile

import numpy as np
import torch

PAGES_PER_CHUNK = 16 * 32  # blocks per chunk × layers


def _store(root: str, drives: int, chunks: int, ctas: int, threads: int):
    from ..models.kv_geometry import LLAMA3_8B as g
    from ..storage.tutti_store import TuttiKVStore

    st = TuttiKVStore(root, g, capacity_chunks=max(16, chunks), mounts=[os.path.join(root, f"nvme{d}") for d in range(drives)],
                      device=0, segment_file_slots=max(4, chunks // drives + 1),
                      runtime_options={"controller_threads": threads, "leases": 64, "max_ctas_per_op": ctas,
                                       "slots_per_lease": 8})
    return st.open(), g


def _restore_rate(st, g, keys, chunks: int, layers: int, iters: int, warmup: int) -> dict:
    nblk = chunks * g.blocks_per_chunk
    dst = (np.arange(nblk) + nblk).reshape(chunks, g.blocks_per_chunk)
    ly = list(range(layers))
    for _ in range(warmup):
        st.get_paged(keys[:chunks], dst, layers=ly).wait()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        st.get_paged(keys[:chunks], dst, layers=ly).wait()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    pages = nblk * layers
    nbytes = pages * g.block_layer_bytes
    prof = st.runtime.last_submit_profile()
    return {"pages": pages, "bytes": nbytes, "ms": round(ms, 3), "GBps": round(nbytes / ms / 1e6, 2),
            "GiBps": round(nbytes / ms * 1e3 / 2**30, 2), "commands": int(prof.get("commands", 0))}


def _fill(st, g, chunks: int):
    from ..index.chunk_index import chunk_keys_for_tokens

    nblk = chunks * g.blocks_per_chunk
    pool = torch.randn(g.pool_shape(2 * nblk + 16), dtype=g.dtype, device="cuda")
    st.register_pool(pool)
    keys = chunk_keys_for_tokens(list(range(chunks * g.chunk_tokens)), g.chunk_tokens, namespace=b"sweep")
    st.put_paged(keys, np.arange(nblk).reshape(chunks, g.blocks_per_chunk)).wait()
    return pool, keys


def shape_for(pages: int) -> tuple[int, int]:
    """(chunks, layers) whose page count is closest to ``pages`` with at most 32 layers."""
    chunks = max(1, math.ceil(pages / PAGES_PER_CHUNK))
    layers = max(1, min(32, round(pages / (16 * chunks))))
    return chunks, layers


def run(args) -> dict:
    root = tempfile.mkdtemp(prefix="tutti_sweep_")
    out = {"bench": "io_sweep", "page_bytes": 65536, "drives": args.drives, "batch": [], "width": []}
    try:
        targets = [int(x) for x in args.batches.split(",")]
        max_chunks = max(shape_for(p)[0] for p in targets)
        st, g = _store(os.path.join(root, "batch"), args.drives, max_chunks, args.ctas, args.threads)
        try:
            pool, keys = _fill(st, g, max_chunks)
            for p in targets:
                c, l = shape_for(p)
                out["batch"].append({"target_pages": p, "ctas": args.ctas,
                                     **_restore_rate(st, g, keys, c, l, args.iters, args.warmup)})
            del pool
        finally:
            st.close()
        c, l = shape_for(args.width_pages)
        for w in [int(x) for x in args.widths.split(",")]:
            st, g = _store(os.path.join(root, f"w{w}"), args.drives, c, w, args.threads)
            try:
                pool, keys = _fill(st, g, c)
                out["width"].append({"ctas": w, "inflight_commands": w * 8,
                                     **_restore_rate(st, g, keys, c, l, args.iters, args.warmup)})
                del pool
            finally:
                st.close()
    finally:
        shutil.rmtree(root, ignore_errors=True)
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--drives", type=int, default=4)
    p.add_argument("--threads", type=int, default=3, help="emulated-controller host threads per drive")
    p.add_argument("--ctas", type=int, default=64, help="max_ctas_per_op of the batch sweep")
    p.add_argument("--batches", default="128,486,972,1944,3888")
    p.add_argument("--width-pages", type=int, default=486)
    p.add_argument("--widths", default="1,2,4,8,16,32,64")
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    args = p.parse_args(argv)
    print(json.dumps(run(args)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
