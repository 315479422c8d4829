"""Microbenchmarks of the sm_100a kernels, each on a case sized for an ncu capture.

    python -m tutti_b200.benchmarks.kernels copy     # batched bulk page copy (HBM -> HBM, 32 KiB pages)
    python -m tutti_b200.benchmarks.kernels fp8      # block-scaled fp8 quantise of bf16 rows
    python -m tutti_b200.benchmarks.kernels hash     # chained BLAKE2b-128 prefix keys
    python -m tutti_b200.benchmarks.kernels checksum # KV block checksums
    python -m tutti_b200.benchmarks.kernels io       # fused NVMe io kernel restore (emulated controllers);
                                                     #   --direction write: store; --async-completion: split launches;
                                                     #   --media memory [--direct-reads]: drive DMA into HBM

Each prints one JSON line: kernel time (CUDA events, after warm-up, inputs
larger than L2 where the kernel is bandwidth-bound) and achieved rates.
``--iters`` sets timed launches; ``--warmup`` untimed ones.
"""
from __future__ import annotations

import os

# Before CUDA starts: emulated drives that DMA into HBM need eager kernel
# loading and enough hardware queues (see the GPU NVMe data path).
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")

import argparse  # noqa: E402
import json  # noqa: E402
import shutil  # noqa: E402
import tempfile  # noqa: E402

import numpy as np  # noqa: E402
import torch  # noqa: E402


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_copy(args) -> dict:
    from .. import ops

    nbytes = args.mib << 20
    page = 32768
    a = torch.empty(nbytes, dtype=torch.uint8, device="cuda").random_()
    b = torch.empty_like(a)
    n = nbytes // page
    src = a.data_ptr() + torch.arange(n, device="cuda", dtype=torch.int64) * page
    dst = b.data_ptr() + torch.randperm(n, device="cuda") * page
    items = torch.stack([src, dst, torch.full_like(src, page)], 1).contiguous()
    from .._native import ops as _ops

    ms = _time(lambda: _ops().copy_items(items, True), args.iters, args.warmup)
    ok = True
    if args.verify:
        ops.page_copy(src[:1], dst[:1], page)
        ok = bool(torch.equal(b[int(dst[0] - b.data_ptr()):][:page], a[:page]))
    return {"kernel": "bulk_copy_kernel", "bytes": nbytes, "ms": ms, "GBps_rw": 2 * nbytes / ms / 1e6,
            "pages": n, "ok": ok}


def bench_fp8(args) -> dict:
    from .._native import ops as _ops

    rows = (args.mib << 20) // 256
    x = torch.randn(rows, 128, dtype=torch.bfloat16, device="cuda")
    q = torch.empty(rows, 128, dtype=torch.uint8, device="cuda")
    ms = _time(lambda: _ops().fp8_quant(x, 128), args.iters, args.warmup)
    moved = x.numel() * 2 + q.numel() + rows * 4
    qq, ss = _ops().fp8_quant(x, 128)
    ms_d = _time(lambda: _ops().fp8_dequant(qq, ss, torch.bfloat16), args.iters, args.warmup)
    return {"kernel": "quant16_bf16_kernel", "rows": rows, "ms": ms, "GBps": moved / ms / 1e6,
            "dequant": {"kernel": "dequant16_bf16_kernel", "ms": ms_d, "GBps": moved / ms_d / 1e6}}


def bench_hash(args) -> dict:
    from .. import ops
    from ..index.chunk_index import chunk_keys_for_tokens

    rng = np.random.default_rng(0)
    reqs = [rng.integers(0, 150000, size=args.tokens).tolist() for _ in range(args.requests)]
    dev_reqs = [torch.tensor(r, dtype=torch.int64, device="cuda") for r in reqs]  # token ids already in HBM
    import time

    t0 = time.perf_counter()
    ops.prefix_hash(dev_reqs, args.chunk)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    for _ in range(args.iters):
        keys = ops.prefix_hash(dev_reqs, args.chunk)
    torch.cuda.synchronize()
    gpu_ms = (time.perf_counter() - t1) / args.iters * 1e3
    t2 = time.perf_counter()
    ref = [chunk_keys_for_tokens(r, args.chunk) for r in reqs]
    cpu_ms = (time.perf_counter() - t2) * 1e3
    return {"kernel": "prefix_hash_kernel", "requests": args.requests, "tokens": args.tokens,
            "gpu_api_ms": gpu_ms, "cpu_hashlib_ms": cpu_ms, "ok": keys == ref, "first_call_ms": (t1 - t0) * 1e3}


def bench_checksum(args) -> dict:
    from .. import ops

    nb = (args.mib << 20) // (2 * 2 * 16 * 8 * 128 * 2)
    pool = torch.randn(2, 2, nb, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
    blocks = torch.arange(nb, device="cuda")
    ms = _time(lambda: ops.kv_checksum(pool, blocks), args.iters, args.warmup)
    nbytes = pool.numel() * 2
    return {"kernel": "checksum_uniform_kernel", "bytes": nbytes, "ms": ms, "GBps": nbytes / ms / 1e6}


def bench_io(args) -> dict:
    from .. import ops
    from ..index.chunk_index import chunk_keys_for_tokens
    from ..models.kv_geometry import LLAMA3_8B as g
    from ..storage.tutti_store import TuttiKVStore

    root = tempfile.mkdtemp(prefix="tutti_kio_")
    try:
        tokens = args.tokens
        nblk = tokens // g.block_size
        nch = tokens // g.chunk_tokens
        st = TuttiKVStore(root, g, capacity_chunks=max(16, 2 * nch), mounts=[os.path.join(root, f"nvme{d}") for d in range(4)],
                          device=0, segment_file_slots=max(4, nch // 2 + 1), stored_format=args.stored_format,
                          runtime_options={"controller_threads": 3, "leases": 64, "max_ctas_per_op": 64,
                                           "slots_per_lease": 8, "async_completion": bool(args.async_completion),
                                           "emulator_media": args.media, "direct_reads": bool(args.direct_reads)})
        st.open()
        nb = 2 * nblk + 64
        pool = torch.randn(g.pool_shape(nb), dtype=g.dtype, device="cuda")
        st.register_pool(pool)
        keys = chunk_keys_for_tokens(list(range(tokens)), g.chunk_tokens)
        src = np.arange(nblk).reshape(nch, g.blocks_per_chunk)
        st.put_paged(keys, src).wait()
        dst = (np.arange(nblk) + nblk).reshape(nch, g.blocks_per_chunk)
        if args.direction == "write":
            # fresh keys every launch: each store writes (and commits) new chunks from the source blocks
            state = {"n": 0}
            kernel_ms = []

            def store_once():
                state["n"] += 1
                k = chunk_keys_for_tokens(list(range(tokens)), g.chunk_tokens, namespace=b"w%d" % state["n"])
                s = torch.cuda.current_stream()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                comp = st.put_paged(k, src, stream=s)
                e1.record(s)
                comp.wait()  # the io kernel, then the commit (write-back, payload and header syncs)
                kernel_ms.append(e0.elapsed_time(e1))
                st.drop(k)  # free the slots for the next launch

            ms = _time(store_once, args.iters, args.warmup)
            nbytes = nblk * g.num_layers * g.block_layer_bytes
            kms = float(np.median(kernel_ms[args.warmup:])) if len(kernel_ms) > args.warmup else float("nan")
            st.close()
            return {"kernel": "nvme_io_kernel", "direction": "write", "stored_format": args.stored_format,
                    "media": args.media, "bytes": nbytes, "kernel_ms": kms, "kernel_GBps": nbytes / kms / 1e6,
                    "ms_with_commit": ms, "GBps_with_commit": nbytes / ms / 1e6, "ok": True}
        ms = _time(lambda: st.get_paged(keys, dst).wait(), args.iters, args.warmup)
        want = pool[:, :, :nblk]
        if args.stored_format == "fp8_block128":
            q, sc = ops.fp8_quant(want.reshape(-1, 128))
            want = ops.fp8_dequant(q, sc).reshape(want.shape)
        ok = bool(torch.equal(pool[:, :, nblk:2 * nblk], want))
        nbytes = nblk * g.num_layers * g.block_layer_bytes
        st.close()
        return {"kernel": "nvme_io_kernel", "direction": "read", "async_completion": bool(args.async_completion),
                "media": args.media, "direct_reads": bool(args.direct_reads),
                "stored_format": args.stored_format, "bytes": nbytes, "ms": ms,
                "GBps": nbytes / ms / 1e6, "ok": ok}
    finally:
        shutil.rmtree(root, ignore_errors=True)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("which", choices=["copy", "fp8", "hash", "checksum", "io"])
    p.add_argument("--mib", type=int, default=1024)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--tokens", type=int, default=4096)
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--chunk", type=int, default=256)
    p.add_argument("--verify", action="store_true")
    p.add_argument("--stored-format", choices=["native", "fp8_block128"], default="native")
    p.add_argument("--direction", choices=["read", "write"], default="read", help="io: restore or store")
    p.add_argument("--async-completion", action="store_true", help="io: split submit / drain launches")
    p.add_argument("--media", choices=["files", "memory"], default="files",
                   help="io: emulated drives' media (memory: copy-engine DMA into HBM)")
    p.add_argument("--direct-reads", action="store_true",
                   help="io: drives DMA reads straight into the pool pages (memory media)")
    args = p.parse_args(argv)
    torch.cuda.set_device(0)
    fn = {"copy": bench_copy, "fp8": bench_fp8, "hash": bench_hash, "checksum": bench_checksum, "io": bench_io}
    print(json.dumps(fn[args.which](args)))


if __name__ == "__main__":
    main()
