"""Multi-GPU restore benchmark: local reads vs drive-affine NVLink fan-out.

Launch one rank per GPU::

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m tutti_b200.benchmarks.fanout --mode tp|mla [--drives D] [--affine 0,1]

``--mode tp``: Llama-3.1-70B KV sliced over N TP ranks; every rank persisted its
own slice of each chunk. ``local`` restores each rank's slice with its own
reads; ``fanout`` has the GPU affine to each drive read every rank's slices on
that drive and store them into the owners' pools over NVLink from the io kernel.

``--mode mla``: DeepSeek-V3 latent cache, identical on every rank, persisted
once by the chunk's replica owner. ``local`` makes every rank read every chunk
(N-fold storage reads); ``fanout`` reads each chunk once and the io kernel
stores it into all N pools.

Each step's device time is taken with CUDA events on every rank, max over
ranks; bytes are the HBM bytes that land in all pools. Restored pools are
compared with the persisted source blocks.
Parity: reference tutti/storage/tutti_nvme/replica_direct.py (owner reads,
peers pull over IPC) and doc/design/replica-sharded-io-allgather.md
(replica dedup throughput).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import shutil
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

from ..index.chunk_index import chunk_keys_for_tokens
from ..models.kv_geometry import DEEPSEEK_V3_MLA, LLAMA3_70B
from ..parallel.fanout import FanoutRestorer, PeerPools, ReadyBoard, RestoreItem, owner_of
from ..common import numa
from ..storage.tutti_store import TuttiKVStore


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--mode", choices=["tp", "mla"], default="tp")
    p.add_argument("--prefix-tokens", type=int, default=16384)
    p.add_argument("--pool-blocks", type=int, default=0, help="0: 2x the prefix")
    p.add_argument("--drives", type=int, default=0, help="0: one per rank")
    p.add_argument("--affine", default="", help="comma list: drive d belongs to GPU affine[d %% len]; default all")
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=2)
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_fanout"))
    p.add_argument("--controller-threads", type=int, default=0)
    p.add_argument("--leases", type=int, default=128)
    p.add_argument("--ctas", type=int, default=64)
    p.add_argument("--ordering", choices=["flags", "barrier"], default="flags",
                   help="order each rank after every rank's share: device ready flags or a host barrier")
    p.add_argument("--store", choices=["local", "fanout"], default="local",
                   help="persist the prefix with each rank's own writes or through the drive-affine GPUs")
    p.add_argument("--stored-format", choices=["native", "fp8_block128"], default="native",
                   help="fp8_block128: the io kernel quantises on store and dequantises on restore")
    p.add_argument("--timing", action="store_true", help="per-command %%globaltimer breakdown of the last mode")
    return p.parse_args(argv)


def main(argv=None) -> int:
    args = parse(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa_bind = numa.bind_to_gpu(local)  # host work on the GPU's node, before any thread or pinned buffer
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    ctl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
    g = (LLAMA3_70B.with_tp(world) if args.mode == "tp" else DEEPSEEK_V3_MLA)
    nblk = args.prefix_tokens // g.block_size
    nchunks = args.prefix_tokens // g.chunk_tokens
    pool_blocks = args.pool_blocks or 2 * nblk
    drives = args.drives or world
    affine = [int(x) for x in args.affine.split(",")] if args.affine else list(range(world))
    if rank == 0:
        shutil.rmtree(args.root, ignore_errors=True)
    dist.barrier(group=ctl)
    mounts = [os.path.join(args.root, f"nvme{d}") for d in range(drives)]
    ncpu = os.cpu_count() or 8
    threads = args.controller_threads or max(1, min(3, (2 * ncpu // world) // max(1, drives)))
    opts = {"controller_threads": threads, "leases": args.leases, "max_ctas_per_op": args.ctas,
            "slots_per_lease": 8, "slot_bytes": 1 << 20, "queue_depth": 256, "mdts_bytes": 1 << 20,
            "timing": bool(args.timing)}
    spf = max(16, (nchunks + drives - 1) // drives)
    store = TuttiKVStore(args.root, g, capacity_chunks=spf * drives, mounts=mounts, device=local,
                         rank=rank, rank_count=world, runtime_options=opts, segment_file_slots=spf,
                         namespace=b"fanout-" + args.mode.encode(), stored_format=args.stored_format)
    store.open()
    pool = torch.zeros(g.pool_shape(pool_blocks), dtype=g.dtype, device=dev)
    store.register_pool(pool)
    peers = PeerPools(pool, group=ctl)
    fan = FanoutRestorer(store, peers, group=ctl)

    # Source: the prefix in the first nblk blocks; every rank knows every rank's (key, blocks).
    tokens = torch.randint(0, 128_000, (args.prefix_tokens,), generator=torch.Generator().manual_seed(11))
    keys = chunk_keys_for_tokens(tokens.tolist(), g.chunk_tokens)
    src = np.arange(nblk).reshape(nchunks, g.blocks_per_chunk)
    gen = torch.Generator(device=dev).manual_seed(100 + (rank if args.mode == "tp" else 0))
    pool[:, :, :nblk] = torch.randn(pool[:, :, :nblk].shape, dtype=g.dtype, device=dev, generator=gen)
    if args.mode == "tp":
        mine = list(range(nchunks))
    else:
        mine = [i for i, k in enumerate(keys) if owner_of(k, world) == rank]
    torch.cuda.synchronize()
    dist.barrier(group=ctl)
    t_store = time.perf_counter()
    if args.store == "fanout":
        src_items = [RestoreItem(rank=r, key=keys[i], block_ids=src[i].tolist()) for r in range(world)
                     for i in range(nchunks) if args.mode == "tp" or owner_of(keys[i], world) == r]
        fan.store(src_items, drives, affine)
    elif mine:
        store.put_paged([keys[i] for i in mine], src[mine]).wait()
    dist.barrier(group=ctl)
    store_ms = (time.perf_counter() - t_store) * 1e3

    # Destination blocks: a seeded permutation of the upper half, one per rank.
    dst = {r: (nblk + np.random.default_rng(r).permutation(pool_blocks - nblk)[:nblk]).reshape(
        nchunks, g.blocks_per_chunk) for r in range(world)}
    items = []
    for r in range(world):
        for i, k in enumerate(keys):
            src_rank = r if args.mode == "tp" else owner_of(k, world)
            items.append(RestoreItem(rank=r, key=k, block_ids=dst[r][i].tolist(), source=src_rank))
    placements = fan.placements({r: sorted({bytes(it.key) for it in items if it.src == r}) for r in range(world)})
    local_items = [it for it in items if it.rank == rank]
    local_pl = [(placements[(it.src, bytes(it.key))][0], placements[(it.src, bytes(it.key))][1]) for it in local_items]
    local_blocks = np.asarray([it.block_ids for it in local_items], dtype=np.int64)
    for path, _ in local_pl:
        store.targets_for([path])
    stream = torch.cuda.current_stream(dev)

    host_ms = {"local": [], "fanout": []}
    board = ReadyBoard(local, group=ctl) if args.ordering == "flags" else None
    epoch = [0]
    pending, tickets = [], []

    def step(mode: str) -> None:
        t0 = time.perf_counter()
        if mode == "local":
            c = store.restore_placements(local_pl, local_blocks, stream=stream)
        else:
            c = fan.restore(items, drives, affine, stream=stream, placements=placements)
        host_ms[mode].append((time.perf_counter() - t0) * 1e3)
        if board is None:
            if c is not None:
                c.wait()
            fan.barrier()  # a pool is whole only once every rank's share has landed
            return
        # device-side: raise this rank's flag behind its share, wait for every rank's
        epoch[0] += 1
        board.signal(0, epoch[0], stream)
        tickets.append(board.wait(0, epoch[0], stream))
        if c is not None:
            pending.append(c)

    def settle() -> None:
        torch.cuda.synchronize()
        for c in pending:
            c.wait()
        pending.clear()
        missing = [board.failed(t) for t in tickets] if board is not None else []
        tickets.clear()
        if any(missing):
            raise RuntimeError(f"ready flags timed out waiting for ranks {missing}")

    def timed(mode: str) -> float:
        for _ in range(args.warmup):
            step(mode)
        settle()
        dist.barrier(group=ctl)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step(mode)
        e1.record(stream)
        settle()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def verify() -> bool:
        s = torch.from_numpy(src.reshape(-1)).to(dev)
        d = torch.from_numpy(dst[rank].reshape(-1)).to(dev)
        want = pool[:, :, s]
        if args.stored_format == "fp8_block128":
            from .. import ops

            q, sc = ops.fp8_quant(want.reshape(-1, 128))
            want = ops.fp8_dequant(q, sc).reshape(want.shape)
        ok = torch.tensor([1.0 if torch.equal(pool[:, :, d], want) else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        return bool(ok.item() == 1.0)

    results = {}
    for mode in ("local", "fanout"):
        pool[:, :, nblk:].zero_()
        torch.cuda.synchronize()
        dist.barrier(group=ctl)
        ms = timed(mode)
        results[mode] = {"ms": round(ms, 3), "verified": verify()}
    hbm_bytes = world * nblk * g.num_layers * g.block_layer_bytes
    # storage bytes read per step: tp reads every slice once either way; mla local reads N copies
    read_bytes = {"local": hbm_bytes, "fanout": hbm_bytes if args.mode == "tp" else hbm_bytes // world}
    for mode, r in results.items():
        r["GBps_into_hbm"] = round(hbm_bytes / (r["ms"] / 1e3) / 1e9, 3)
        r["storage_bytes_per_step"] = read_bytes[mode]
        r["host_submit_ms_p50"] = round(float(np.median(host_ms[mode])), 3)
    timing = store.runtime.io_timing() if args.timing else None
    peers_stats = store.runtime.controller_stats()
    dist.barrier(group=ctl)
    # teardown: nobody reads a peer pool after this barrier
    store.close()
    peers.close()
    if board is not None:
        board.close()
    dist.barrier(group=ctl)
    ok = all(r["verified"] for r in results.values())
    if rank == 0:
        print(json.dumps({"bench": "fanout", "mode": args.mode, "n_gpus": world, "numa_bind": numa_bind, "model": g.fingerprint(),
                          "prefix_tokens": args.prefix_tokens, "drives": drives, "affine_gpus": affine,
                          "steps": args.steps, "warmup": args.warmup, "ordering": args.ordering, "results": results,
                          "store": {"mode": args.store, "wall_ms": round(store_ms, 1)},
                          "controllers": len(peers_stats), "ok": ok, "io_timing": timing}))
    del pool
    dist.destroy_process_group()
    if rank == 0:
        shutil.rmtree(args.root, ignore_errors=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
