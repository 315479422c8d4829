"""Restore throughput and compute slowdown while an SM-filling kernel runs.

    python -m tutti_b200.benchmarks.interference [--compute gemm|fma] [--prefix-tokens 32768]
                                                 [--layerwise] [--drives 4]

A compute workload runs on its own stream (a loop of cuBLAS bf16 GEMMs that
fill every SM, or this package's persistent FMA kernel) while restores of a
Llama-3.1-8B prefix run back to back on an io stream. Three modes:

* ``none``:  compute alone (its duration is the baseline);
* ``sync``:  each restore is one io-kernel launch whose CTAs stay resident
  from the first command to the last (the queue engine polls CQs on the SMs);
* ``split``: each restore is a one-warp-per-lease submit launch that queues
  the commands and exits, and a drain launch that the host issues once the
  drives have posted every CQE of the op (read from the host-resident CQs),
  which then only moves the data (async_completion; 64 x 64 HBM slots hold a
  whole 32 k-token prefix).

Reported per mode: compute time (CUDA events on the compute stream) and its
slowdown against ``none``, restore GB/s over the compute window, and the
restores that finished in it. Drives: memory media, DMA into HBM staging.

Parity: reference examples/nvme_bw_probe/async_completion_bench (persistent
compute kernel + restores; doc/design/async-nvme-completion.md:444-508 reports
compute +31-34 % sync vs +0.0 % async on H20).
"""
from __future__ import annotations

import os

os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")

import argparse  # noqa: E402
import json  # noqa: E402
import shutil  # noqa: E402
import tempfile  # noqa: E402
import time  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--compute", choices=["gemm", "fma"], default="gemm")
    p.add_argument("--compute-ms", type=float, default=600.0, help="target duration of the compute run alone")
    p.add_argument("--fma-blocks-per-sm", type=int, default=4)
    p.add_argument("--prefix-tokens", type=int, default=32768)
    p.add_argument("--pool-blocks", type=int, default=16384)
    p.add_argument("--drives", type=int, default=4)
    p.add_argument("--ctas", type=int, default=32)
    p.add_argument("--slots", type=int, default=16)
    p.add_argument("--layerwise", action="store_true", help="one restore op per layer instead of per prefix")
    p.add_argument("--split-ctas", type=int, default=64, help="split mode: CTAs (leases) per op")
    p.add_argument("--split-slots", type=int, default=64, help="split mode: HBM slots per CTA")
    p.add_argument("--drain-after-us", type=int, default=500000,
                   help="split mode: latest drain launch; it normally starts once the drives posted every CQE")
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_interference"))
    return p.parse_args(argv)


def _compute_fn(args, dev):
    if args.compute == "gemm":
        a = torch.randn(8192, 8192, dtype=torch.bfloat16, device=dev)
        b = torch.randn(8192, 8192, dtype=torch.bfloat16, device=dev)
        c = torch.empty(8192, 8192, dtype=torch.bfloat16, device=dev)

        def one(n):
            for _ in range(n):
                torch.matmul(a, b, out=c)
        return one
    from .._native import ops as _ops

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    out = torch.empty(sms * args.fma_blocks_per_sm * 256, dtype=torch.float32, device=dev)

    def one(n):
        _ops().persistent_fma(out, 4096 * n, args.fma_blocks_per_sm)
    return one


def main(argv=None) -> int:
    args = parse(argv)
    from ..index.chunk_index import chunk_keys_for_tokens
    from ..models.kv_geometry import LLAMA3_8B
    from ..storage.tutti_store import TuttiKVStore

    g = LLAMA3_8B
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nblk = args.prefix_tokens // g.block_size
    nchunks = args.prefix_tokens // g.chunk_tokens
    spf = max(16, (nchunks + args.drives - 1) // args.drives)
    pool = torch.empty(g.pool_shape(args.pool_blocks), dtype=g.dtype, device=dev)
    rng = np.random.default_rng(0)
    src = rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, g.blocks_per_chunk)
    pool.normal_()
    keys = chunk_keys_for_tokens(list(range(args.prefix_tokens)), g.chunk_tokens, namespace=b"interference")
    shutil.rmtree(args.root, ignore_errors=True)
    stores = {}
    for mode, split in (("sync", False), ("split", True)):
        root = os.path.join(args.root, mode)
        ctas, slots = (args.split_ctas, args.split_slots) if split else (args.ctas, args.slots)
        opts = {"emulator_media": "memory", "controller_threads": 1, "leases": 2 * ctas,
                "max_ctas_per_op": ctas, "slots_per_lease": slots, "queue_depth": 1024,
                "image_budget_bytes": spf * (g.chunk_bytes + (128 << 10)) + (128 << 20),
                "async_completion": split, "async_fallback_us": args.drain_after_us}
        st = TuttiKVStore(root, g, capacity_chunks=spf * args.drives,
                          mounts=[os.path.join(root, f"nvme{d}") for d in range(args.drives)], device=0,
                          runtime_options=opts, segment_file_slots=spf, namespace=b"interference")
        st.open()
        st.register_pool(pool)
        st.put_paged(keys, src).wait()
        stores[mode] = st
    ref = pool[:, :, torch.from_numpy(src.reshape(-1)).to(dev)].clone()

    compute = _compute_fn(args, dev)
    cstream, io = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # calibrate: units of compute that last about --compute-ms alone
    with torch.cuda.stream(cstream):
        compute(2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cstream)
    with torch.cuda.stream(cstream):
        compute(10)
    e1.record(cstream)
    torch.cuda.synchronize()
    units = max(1, int(args.compute_ms / (e0.elapsed_time(e1) / 10)))

    def restore_op(st, perm):
        if not args.layerwise:
            return [st.get_paged(keys, perm, stream=io)]
        return [st.get_paged(keys, perm, layers=[layer], stream=io) for layer in range(g.num_layers)]

    results = {}
    for mode in ("none", "sync", "split", "none"):
        st = stores.get(mode)
        if st is not None:  # warm the path
            for c in restore_op(st, rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, g.blocks_per_chunk)):
                c.wait()
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(cstream)
        with torch.cuda.stream(cstream):
            compute(units)
        c1.record(cstream)
        done_bytes, restores, last_perm = 0, 0, None
        t0 = time.perf_counter()
        if st is not None:
            pending = []
            while not c1.query():
                perm = rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, g.blocks_per_chunk)
                pending.append((perm, restore_op(st, perm)))
                while len(pending) >= 2:
                    p, comps = pending.pop(0)
                    for c in comps:
                        c.wait()
                    done_bytes += nblk * g.num_layers * g.block_layer_bytes
                    restores += 1
                    last_perm = p
            io_s = time.perf_counter() - t0
            for p, comps in pending:
                for c in comps:
                    c.wait()
                last_perm = p
        else:
            io_s = 0.0
        torch.cuda.synchronize()
        ms = c0.elapsed_time(c1)
        row = {"compute_ms": round(ms, 2)}
        if st is not None:
            ok = bool(torch.equal(pool[:, :, torch.from_numpy(last_perm.reshape(-1)).to(dev)], ref))
            row.update({"restores_in_window": restores, "io_GBps": round(done_bytes / io_s / 1e9, 2) if io_s else None,
                        "verified": ok})
        results[mode if mode not in results else "none_after"] = row
    base = (results["none"]["compute_ms"] + results["none_after"]["compute_ms"]) / 2
    for mode in ("sync", "split"):
        results[mode]["compute_slowdown_pct"] = round(100.0 * (results[mode]["compute_ms"] / base - 1.0), 1)
    for st in stores.values():
        st.close()
    shutil.rmtree(args.root, ignore_errors=True)
    print(json.dumps({"bench": "interference", "compute": args.compute, "layerwise": args.layerwise,
                      "compute_units": units, "prefix_tokens": args.prefix_tokens, "drives": args.drives,
                      "ctas": args.ctas, "slots": args.slots, "split_ctas": args.split_ctas,
                      "split_slots": args.split_slots, "results": results}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
