"""Serving-trace benchmark: long-prefix reuse restored from SSD under Poisson arrivals.

Launch one rank per GPU (TP = number of ranks)::

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m tutti_b200.benchmarks.serving_trace [--requests 48] [--restore fanout|local]

Trace (seeded, identical on every rank): prefix-reuse probability 0.8 with a
Zipf(1.1) choice over 512 distinct prefixes, otherwise a new prefix; prefix
lengths uniform in [8k, 64k] tokens times ``--length-scale`` (default 1/8 so
that the touched prefixes fit the GPU box's page cache; 1.0 is the full
config); 256 output tokens. KV shape: Llama-3.1-70B (80 layers, 8 KV heads,
head_dim 128, bf16, block 16) sliced over the TP ranks.

Every request runs for real through the store: a prefix hit is restored from
the emulated NVMe drives into the paged pool (``fanout``: the GPU affine to
each drive reads it for all ranks and its io kernel stores every rank's slice
over NVLink; ``local``: each rank reads its own slice), timed on the device
and taken as the max over ranks; the uncached remainder is persisted after its
(modelled) prefill. Nothing is kept in HBM between requests, so every reuse is
an SSD restore.

Prefill (``--prefill run``, the default) runs for real: a random-init
Llama-3.1-70B sharded over the TP ranks (``models.llama.LlamaModel``: sharded
heads and MLP, NCCL all-reduce after the row-parallel GEMMs) prefills each
request's uncached tokens after its restored prefix, attending over the
restored KV in the paged pool, and the new chunks it writes are what gets
persisted; the recompute baseline prefills the whole prompt. Both are
CUDA-event timed, max over ranks. ``--prefill model`` instead models prefill
as FLOPs / (sustained bf16 peak x ``--mfu``). Decode is modelled as 256 steps
of reading the rank's weights at the measured HBM bandwidth, and continuous
batching is assumed so that only prefills queue. TTFT at each arrival rate
(0.5, 1, 2, 4 req/s) is the FIFO wait plus the request's restore and prefill.
Parity: reference scripts/vllm/vllm_profile_offline.py (--tokens, --reuse-pct)
and doc/design/kv-storage-layout-and-io-submission.md (A/B request latency).
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

from .. import ops
from ..index.chunk_index import chunk_keys_for_tokens
from ..models.kv_geometry import LLAMA3_70B
from ..models.llama import LLAMA_3_1_70B, LlamaModel
from ..parallel.fanout import FanoutRestorer, PeerPools, RestoreItem
from ..common import numa
from ..storage.tutti_store import TuttiKVStore

PARAMS_70B = 70.6e9
HIDDEN_70B = 8192
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops_sustained": 1400.0}


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--requests", type=int, default=48)
    p.add_argument("--distinct", type=int, default=512)
    p.add_argument("--reuse", type=float, default=0.8)
    p.add_argument("--zipf", type=float, default=1.1)
    p.add_argument("--min-prefix", type=int, default=8192)
    p.add_argument("--max-prefix", type=int, default=65536)
    p.add_argument("--length-scale", type=float, default=0.125)
    p.add_argument("--output-tokens", type=int, default=256)
    p.add_argument("--rates", default="0.5,1,2,4")
    p.add_argument("--restore", choices=["fanout", "local"], default="fanout")
    p.add_argument("--drives", type=int, default=0, help="0: one per rank")
    p.add_argument("--affine", default="", help="drive d belongs to GPU affine[d %% len]; default all ranks")
    p.add_argument("--warm", type=int, default=16,
                   help="persist the N most popular prefixes before the trace (a warm SSD cache)")
    p.add_argument("--mfu", type=float, default=0.5, help="--prefill model: fraction of the sustained bf16 peak")
    p.add_argument("--prefill", choices=["run", "model"], default="run",
                   help="run: a random-init 70B TP prefill on the GPUs; model: FLOPs at --mfu")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_trace"))
    p.add_argument("--leases", type=int, default=128)
    p.add_argument("--ctas", type=int, default=64)
    return p.parse_args(argv)


def peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])),
                "source": "measured"}
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def prefix_lengths(args, chunk: int) -> np.ndarray:
    """Token length of each distinct prefix (prefix id = Zipf popularity rank - 1)."""
    rng = np.random.default_rng(args.seed + 7)
    lo, hi = int(args.min_prefix * args.length_scale), int(args.max_prefix * args.length_scale)
    return (rng.integers(lo, hi + 1, args.distinct) // chunk).clip(1) * chunk


def make_trace(args, chunk: int) -> list[dict]:
    """Seeded request list: prefix id, prefix tokens (chunk multiple), whether it reuses a prefix."""
    rng = np.random.default_rng(args.seed)
    ranks = np.arange(1, args.distinct + 1, dtype=np.float64)
    zipf = ranks ** -args.zipf
    zipf /= zipf.sum()
    lo, hi = int(args.min_prefix * args.length_scale), int(args.max_prefix * args.length_scale)
    lengths = prefix_lengths(args, chunk)
    out, fresh = [], args.distinct
    for _ in range(args.requests):
        if rng.random() < args.reuse:
            pid = int(rng.choice(args.distinct, p=zipf))
            length = int(lengths[pid])
        else:
            pid = fresh
            fresh += 1
            length = int((rng.integers(lo, hi + 1) // chunk) * chunk) or chunk
        out.append({"prefix": pid, "tokens": length})
    return out


def prefix_tokens(pid: int, n: int) -> list[int]:
    return np.random.default_rng(10_000 + pid).integers(0, 128_000, n).tolist()


def prefill_seconds(new_tokens: int, ctx_tokens: int, tp: int, pk: dict, mfu: float) -> float:
    """Modelled prefill of ``new_tokens`` after ``ctx_tokens`` cached ones, per TP rank."""
    if new_tokens <= 0:
        return 0.0
    dense = 2.0 * PARAMS_70B * new_tokens
    attn = 4.0 * 80 * HIDDEN_70B * new_tokens * (ctx_tokens + new_tokens / 2)
    return (dense + attn) / tp / (pk["bf16_tflops_sustained"] * 1e12 * mfu)


def main(argv=None) -> int:
    args = parse(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa_bind = numa.bind_to_gpu(local)  # host work on the GPU's node, before any thread or pinned buffer
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    ctl = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=600))
    g = LLAMA3_70B.with_tp(world)
    trace = make_trace(args, g.chunk_tokens)
    drives = args.drives or world
    affine = [int(x) for x in args.affine.split(",")] if args.affine else list(range(world))
    if rank == 0:
        shutil.rmtree(args.root, ignore_errors=True)
    dist.barrier(group=ctl)
    ncpu = os.cpu_count() or 8
    threads = max(1, min(3, (2 * ncpu // world) // max(1, drives)))
    opts = {"controller_threads": threads, "leases": args.leases, "max_ctas_per_op": args.ctas,
            "slots_per_lease": 8, "slot_bytes": 1 << 20, "queue_depth": 256, "mdts_bytes": 1 << 20}
    distinct_tokens = {}
    for r in trace:
        distinct_tokens[r["prefix"]] = r["tokens"]
    warm = [{"prefix": pid, "tokens": int(t)} for pid, t in enumerate(prefix_lengths(args, g.chunk_tokens)[:args.warm])]
    for r in warm:
        distinct_tokens[r["prefix"]] = r["tokens"]
    chunks_total = sum(t // g.chunk_tokens for t in distinct_tokens.values())
    spf = 64
    cap = ((chunks_total + spf * drives - 1) // (spf * drives) + 1) * spf * drives
    store = TuttiKVStore(args.root, g, capacity_chunks=cap,
                         mounts=[os.path.join(args.root, f"nvme{d}") for d in range(drives)], device=local,
                         rank=rank, rank_count=world, runtime_options=opts, segment_file_slots=spf,
                         namespace=b"trace")
    store.open()
    store.layout.precreate_until(cap)  # materialise the segment files up front (untimed setup)
    max_blocks = max(r["tokens"] for r in trace + warm) // g.block_size
    pool = torch.zeros(g.pool_shape(2 * max_blocks), dtype=g.dtype, device=dev)
    store.register_pool(pool)
    peers = PeerPools(pool, group=ctl)
    fan = FanoutRestorer(store, peers, group=ctl)
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    rng = np.random.default_rng(args.seed + 1)

    def mx(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model = None
    if args.prefill == "run":
        model = LlamaModel(LLAMA_3_1_70B, dev, seed=3, tp_rank=rank, tp_size=world)
        # load the prefill's kernels before any restore is in flight (a lazily loaded
        # kernel waits for the running io kernel)
        model.prefill([torch.zeros(g.chunk_tokens, dtype=torch.long)], [0], [torch.arange(g.blocks_per_chunk)], pool)
        torch.cuda.synchronize()

    def run_prefill(tokens: list[int], cached: int, table: np.ndarray) -> float:
        """Device ms (max over ranks) of prefilling ``tokens[cached:]`` after ``cached`` tokens."""
        new = torch.tensor(tokens[cached:], dtype=torch.long)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        model.prefill([new], [cached], [torch.from_numpy(table.reshape(-1))], pool)
        e1.record(stream)
        torch.cuda.synchronize()
        return mx(e0.elapsed_time(e1))

    records = []
    gen = torch.Generator(device=dev).manual_seed(rank)
    digests: dict[bytes, torch.Tensor] = {}  # this rank's slice of every persisted chunk
    mismatches = 0
    # warm cache: the most popular prefixes are already on SSD when the trace starts
    for r in warm:
        keys = chunk_keys_for_tokens(prefix_tokens(r["prefix"], r["tokens"]), g.chunk_tokens)
        blocks = np.arange(len(keys) * g.blocks_per_chunk).reshape(len(keys), -1)
        bidx = torch.from_numpy(blocks.reshape(-1)).to(dev)
        pool[:, :, bidx] = torch.randn((g.num_layers, g.planes, bidx.numel()) + tuple(pool.shape[3:]), dtype=g.dtype,
                                       device=dev, generator=gen)
        store.put_paged(keys, blocks).wait()
        dg = ops.kv_checksum(pool, bidx).cpu().reshape(len(keys), g.blocks_per_chunk, g.num_layers, g.planes)
        for c, k in enumerate(keys):
            digests[k] = dg[c]
    dist.barrier(group=ctl)

    for i, req in enumerate(trace):
        n = req["tokens"]
        keys = chunk_keys_for_tokens(prefix_tokens(req["prefix"], n), g.chunk_tokens)
        # cached prefix = what every rank holds (min over ranks)
        hit_local = store.contains_prefix(keys)
        t = torch.tensor([hit_local], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=ctl)
        hit = int(t.item())
        blocks = rng.permutation(pool.shape[2])[: len(keys) * g.blocks_per_chunk].reshape(len(keys), -1)
        restore_ms = 0.0
        if hit:
            fan.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            if args.restore == "fanout":
                items = [RestoreItem(rank=r, key=keys[c], block_ids=blocks[c].tolist()) for r in range(world)
                         for c in range(hit)]
                comp = fan.restore(items, drives, affine, stream=stream)
            else:
                comp = store.get_paged(keys[:hit], blocks[:hit], stream=stream)
            if comp is not None:
                comp.wait()
            fan.barrier()
            e1.record(stream)
            torch.cuda.synchronize()
            restore_ms = mx(e0.elapsed_time(e1))
            got = ops.kv_checksum(pool, torch.from_numpy(blocks[:hit].reshape(-1)).to(dev)).cpu()
            got = got.reshape(hit, g.blocks_per_chunk, *got.shape[1:])
            mismatches += sum(int(not torch.equal(got[c], digests[keys[c]])) for c in range(hit))
        write_ms = 0.0
        prefill_ms = recompute_ms = None
        toks = prefix_tokens(req["prefix"], n)
        if model is not None:
            # the uncached tokens (at least the last one, whose logits start decoding)
            prefill_ms = run_prefill(toks, min(hit * g.chunk_tokens, n - 1), blocks)
        if hit < len(keys):
            # the prefill produced the remaining chunks (modelled: random KV); persist them
            nb = (len(keys) - hit) * g.blocks_per_chunk
            bidx = torch.from_numpy(blocks[hit:].reshape(-1)).to(dev)
            if model is None:
                pool[:, :, bidx] = torch.randn((g.num_layers, g.planes, nb) + tuple(pool.shape[3:]), dtype=g.dtype,
                                               device=dev, generator=gen)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if args.restore == "fanout":
                items = [RestoreItem(rank=r, key=keys[c], block_ids=blocks[c].tolist()) for r in range(world)
                         for c in range(hit, len(keys))]
                fan.store(items, drives, affine)
            else:
                store.put_paged(keys[hit:], blocks[hit:]).wait()
            dist.barrier(group=ctl)
            write_ms = mx((time.perf_counter() - t0) * 1e3)
            dg = ops.kv_checksum(pool, bidx).cpu().reshape(len(keys) - hit, g.blocks_per_chunk, g.num_layers, g.planes)
            for c in range(hit, len(keys)):
                digests[keys[c]] = dg[c - hit]
        if model is not None:
            recompute_ms = run_prefill(toks, 0, blocks)  # the same prompt without the store
        hit_tokens = hit * g.chunk_tokens
        records.append({"tokens": n, "hit_tokens": hit_tokens, "restore_ms": restore_ms, "write_ms": write_ms,
                        "restore_bytes": world * hit * g.blocks_per_chunk * g.num_layers * g.block_layer_bytes,
                        "prefill_s": prefill_ms / 1e3 if prefill_ms is not None
                        else prefill_seconds(n - hit_tokens, hit_tokens, world, pk, args.mfu),
                        "prefill_full_s": recompute_ms / 1e3 if recompute_ms is not None
                        else prefill_seconds(n, 0, world, pk, args.mfu)})

    store.close()
    peers.close()
    del model
    bad = torch.tensor([mismatches], dtype=torch.int64)
    dist.all_reduce(bad, group=ctl)
    ok = int(bad.item()) == 0
    if rank == 0:
        arr_rng = np.random.default_rng(args.seed + 2)
        svc = np.array([r["restore_ms"] / 1e3 + r["prefill_s"] for r in records])
        svc_recompute = np.array([r["prefill_full_s"] for r in records])
        rates = [float(x) for x in args.rates.split(",")]
        gaps = arr_rng.exponential(1.0, len(records))

        def ttft(service: np.ndarray, rate: float) -> np.ndarray:
            arrive = np.cumsum(gaps / rate)
            end, out = 0.0, []
            for a, s in zip(arrive, service):
                start = max(a, end)
                end = start + s
                out.append(end - a)
            return np.asarray(out)

        per_rate = {}
        for rt in rates:
            t_ssd, t_rec = ttft(svc, rt), ttft(svc_recompute, rt)
            per_rate[str(rt)] = {"ttft_p50_s": round(float(np.median(t_ssd)), 4),
                                 "ttft_p90_s": round(float(np.percentile(t_ssd, 90)), 4),
                                 "recompute_ttft_p50_s": round(float(np.median(t_rec)), 4)}
        hits = [r for r in records if r["hit_tokens"]]
        rest_bytes = sum(r["restore_bytes"] for r in hits)
        rest_s = sum(r["restore_ms"] for r in hits) / 1e3
        decode_s = args.output_tokens * (2 * PARAMS_70B / world) / (pk["hbm_gbs"] * 1e9)
        out = {"bench": "serving_trace", "n_gpus": world, "tp": world, "restore": args.restore, "numa_bind": numa_bind,
               "model": g.fingerprint(), "requests": len(records),
               "prefix_tokens": [int(args.min_prefix * args.length_scale), int(args.max_prefix * args.length_scale)],
               "length_scale": args.length_scale, "reuse": args.reuse, "zipf": args.zipf,
               "distinct": args.distinct, "warm_prefixes": args.warm, "hit_requests": len(hits),
               "restore_GBps": round(rest_bytes / rest_s / 1e9, 3) if rest_s else None,
               "restore_ms_p50": round(float(np.median([r["restore_ms"] for r in hits])), 3) if hits else None,
               "write_GBps": round(sum(world * (r["tokens"] - r["hit_tokens"]) // g.block_size * g.num_layers
                                       * g.block_layer_bytes for r in records)
                                   / max(1e-9, sum(r["write_ms"] for r in records) / 1e3) / 1e9, 3),
               "ttft": per_rate, "decode_model_s": round(decode_s, 3), "prefill": args.prefill,
               "prefill_ms_p50": round(float(np.median([r["prefill_s"] for r in records])) * 1e3, 2),
               "recompute_prefill_ms_p50": round(float(np.median([r["prefill_full_s"] for r in records])) * 1e3, 2),
               "compute_model": {"mfu": args.mfu, "peaks": pk} if args.prefill == "model" else None,
               "restored_chunks_mismatched": int(bad.item()),
               "ok": ok}
        print(json.dumps(out))
    del pool
    dist.destroy_process_group()
    if rank == 0:
        shutil.rmtree(args.root, ignore_errors=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
