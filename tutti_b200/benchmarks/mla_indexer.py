"""DeepSeek-V3-shaped MLA latent cache + fp8 indexer cache: store and restore.

    python -m tutti_b200.benchmarks.mla_indexer [--prefix-tokens 65536] [--latent-format fp8_block128]

Two caches per prefix, persisted as separate objects in two namespaces:
  * the latent cache, 61 layers x 576 bf16 values per token (512 latent + 64
    RoPE), block 64 tokens; stored either as is (``native``) or quantised by the
    io kernel to E4M3 with one fp32 scale per 128 values (``fp8_block128``,
    33/64 of the bytes) and dequantised on restore;
  * the indexer cache, 61 layers x 132 bytes per token (128 E4M3 values + one
    fp32 scale), block 64: 8,448-byte pages, which the data path packs into
    LBA-aligned commands.
Values are Gaussian from a seed. Each step restores both caches of the prefix
into seeded random blocks of the paged pools (device time, CUDA events); the
restored latent is checked against the standalone block-scaling kernels and
fp32 (E4M3 bound), the indexer cache byte for byte.

Also measures ``open_batch`` over 500 per-layer files (parallel FIEMAP) against
500 serial ``open`` calls on a fresh runtime.
Parity: reference README.md:23 (batch open of 500 files) and
tutti/storage/tutti_nvme/layerwise_direct.py (per-entity page geometry for the
main KV and the index cache).
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import time

import numpy as np
import torch

from .._native import core
from ..index.chunk_index import chunk_keys_for_tokens
from ..models.kv_geometry import DEEPSEEK_V3_INDEXER, DEEPSEEK_V3_MLA
from ..storage.tutti_store import TuttiKVStore


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--prefix-tokens", type=int, default=65536)
    p.add_argument("--latent-format", choices=["native", "fp8_block128"], default="fp8_block128")
    p.add_argument("--drives", type=int, default=4)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--files", type=int, default=500, help="files for the open_batch measurement")
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_mla"))
    p.add_argument("--leases", type=int, default=192)
    p.add_argument("--ctas", type=int, default=96)
    return p.parse_args(argv)


def open_batch_vs_serial(root: str, n_files: int, opts: dict) -> dict:
    """open_batch over ``n_files`` fresh files vs one open() per file (each on a fresh runtime)."""
    d = os.path.join(root, "openbatch")
    os.makedirs(d, exist_ok=True)
    paths = []
    block = b"\0" * (1 << 20)
    for i in range(n_files):
        p = os.path.join(d, f"layer{i:04d}.seg")
        with open(p, "wb") as f:
            f.write(block)
            f.flush()
            os.fsync(f.fileno())
        paths.append(p)
    uris = ["file://" + p for p in paths]
    best = {"serial": float("inf"), "batch": float("inf")}
    # alternate the two modes twice on fresh runtimes; keep each mode's best
    for mode in ("batch", "serial", "batch", "serial"):
        rt = core().make_emulated_nvme_runtime(0, [d], dict(opts, mapping="fiemap", leases=8, max_ctas_per_op=8))
        t0 = time.perf_counter()
        if mode == "batch":
            hs = rt.open_batch(uris)
        else:
            hs = [rt.open(u) for u in uris]
        best[mode] = min(best[mode], (time.perf_counter() - t0) * 1e3)
        assert len(hs) == n_files
        rt.shutdown(10_000)
    out = {f"{m}_ms": round(v, 2) for m, v in best.items()}
    out["files"] = n_files
    out["speedup"] = round(out["serial_ms"] / max(out["batch_ms"], 1e-6), 2)
    return out


def main(argv=None) -> int:
    args = parse(argv)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    shutil.rmtree(args.root, ignore_errors=True)
    ncpu = os.cpu_count() or 8
    threads = max(1, min(3, (2 * ncpu) // max(1, args.drives)))
    opts = {"controller_threads": threads, "leases": args.leases, "max_ctas_per_op": args.ctas,
            "slots_per_lease": 8, "slot_bytes": 1 << 20, "queue_depth": 256, "mdts_bytes": 1 << 20}
    ob = open_batch_vs_serial(args.root, args.files, opts)

    lat_g, idx_g = DEEPSEEK_V3_MLA, DEEPSEEK_V3_INDEXER
    nblk = args.prefix_tokens // lat_g.block_size
    nchunks = args.prefix_tokens // lat_g.chunk_tokens
    pool_blocks = 2 * nblk
    spf = max(16, (nchunks + args.drives - 1) // args.drives)
    stores, pools = {}, {}
    for name, g, fmt in (("latent", lat_g, args.latent_format), ("indexer", idx_g, "native")):
        root = os.path.join(args.root, name)
        st = TuttiKVStore(root, g, capacity_chunks=spf * args.drives,
                          mounts=[os.path.join(root, f"nvme{d}") for d in range(args.drives)], device=0,
                          runtime_options=opts, segment_file_slots=spf, stored_format=fmt)
        st.open()
        pool = torch.zeros(g.pool_shape(pool_blocks), dtype=g.dtype, device=dev)
        st.register_pool(pool)
        stores[name], pools[name] = st, pool
    gen = torch.Generator(device=dev).manual_seed(0)
    lat = pools["latent"]
    lat[:, :, :nblk] = torch.randn(lat[:, :, :nblk].shape, dtype=lat.dtype, device=dev, generator=gen)
    idx = pools["indexer"]
    # indexer pages: 128 E4M3 values per token, then the per-token fp32 scales (random bytes stand in)
    idx[:, :, :nblk] = torch.randint(0, 256, idx[:, :, :nblk].shape, dtype=torch.uint8, device=dev, generator=gen)
    tokens = torch.randint(0, 128_000, (args.prefix_tokens,), generator=torch.Generator().manual_seed(5)).tolist()
    keys = chunk_keys_for_tokens(tokens, lat_g.chunk_tokens)
    src = np.arange(nblk).reshape(nchunks, lat_g.blocks_per_chunk)
    t0 = time.perf_counter()
    comps = [stores[n].put_paged(keys, src) for n in ("latent", "indexer")]
    for c in comps:
        c.wait()
    store_s = time.perf_counter() - t0
    stored_bytes = sum(sum(x["write_bytes"] for x in stores[n].runtime.controller_stats()) for n in stores)
    ref_lat = lat[:, :, :nblk].clone()
    ref_idx = idx[:, :, :nblk].clone()
    rng = np.random.default_rng(3)
    perms = [nblk + rng.permutation(pool_blocks - nblk)[:nblk].reshape(nchunks, lat_g.blocks_per_chunk)
             for _ in range(args.warmup + args.steps)]
    stream = torch.cuda.current_stream(dev)

    def step(i: int) -> None:
        cs = [stores[n].get_paged(keys, perms[i], stream=stream) for n in ("latent", "indexer")]
        for c in cs:
            c.wait()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.warmup, args.warmup + args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps

    last = torch.from_numpy(perms[-1].reshape(-1)).to(dev)
    got_lat = lat[:, :, last]
    if args.latent_format == "fp8_block128":
        from .. import ops

        rows = ref_lat.reshape(-1, 128)
        q, s = ops.fp8_quant(rows)
        want = ops.fp8_dequant(q, s).reshape(ref_lat.shape)
        amax = rows.float().abs().amax(dim=1, keepdim=True)
        lat_ok = bool(torch.equal(got_lat, want)) and bool(
            torch.all((got_lat.float().reshape(-1, 128) - rows.float()).abs() <= amax / 16 + 1e-6))
    else:
        lat_ok = bool(torch.equal(got_lat, ref_lat))
    idx_ok = bool(torch.equal(idx[:, :, last], ref_idx))
    hbm_bytes = nblk * lat_g.num_layers * (lat_g.block_layer_bytes + idx_g.block_layer_bytes)
    read_bytes = nblk * lat_g.num_layers * (stores["latent"].stored["block_layer_bytes"] + idx_g.block_layer_bytes)
    for st in stores.values():
        st.close()
    shutil.rmtree(args.root, ignore_errors=True)
    out = {"bench": "mla_indexer", "prefix_tokens": args.prefix_tokens, "latent_format": args.latent_format,
           "drives": args.drives, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
           "GBps_into_hbm": round(hbm_bytes / (ms / 1e3) / 1e9, 3),
           "GBps_from_storage": round(read_bytes / (ms / 1e3) / 1e9, 3),
           "hbm_bytes_per_step": hbm_bytes, "storage_bytes_per_step": read_bytes,
           "store_s": round(store_s, 3), "stored_bytes": stored_bytes,
           "latent_ok": lat_ok, "indexer_ok": idx_ok, "open_batch": ob}
    print(json.dumps(out))
    return 0 if (lat_ok and idx_ok) else 1


if __name__ == "__main__":
    sys.exit(main())
