"""p50 TTFT with long-prefix reuse on one GPU (layerwise restore overlapped with prefill).

Workload: random-init Llama-3.1-8B (bf16), a batch of 8 requests, each with a
32,768-token prefix already persisted in the store plus 512 new prompt tokens.
Three ways to produce the first token:
  * ``layerwise``: the KV engine restores layer l+1 on a high-priority IO
    stream while layer l's prefill runs (device-side per-layer events);
  * ``restore_then_prefill``: restore all layers, then prefill (no overlap);
  * ``recompute``: prefill the full 32,768 + 512 tokens (no reuse).
TTFT = CUDA-event time on the compute stream from the batch's arrival (before
the prefix lookup) to the logits of the last prompt token, p50 over iterations.

    python -m tutti_b200.benchmarks.ttft [--requests 8] [--prefix 32768] [--new 512]
"""
from __future__ import annotations

import os

# Before CUDA starts: the emulated drives' in-process DMA needs eager kernel
# loading and enough hardware queues (see the GPU NVMe data path).
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")

import argparse
import json
import shutil
import statistics
import sys
import time

import numpy as np
import torch


def run(args) -> dict:
    from ..engine.core import KVEngine
    from ..index.chunk_index import chunk_keys_for_tokens
    from ..models.llama import LLAMA_3_1_8B, LlamaConfig, LlamaModel
    from ..storage.tutti_store import TuttiKVStore

    dev = torch.device("cuda", args.device)
    torch.cuda.set_device(dev)
    cfg = LLAMA_3_1_8B if args.layers == 32 else LlamaConfig(layers=args.layers)
    g = cfg.geometry()
    R, P, N = args.requests, args.prefix, args.new
    bs = g.block_size
    blocks_per_req = (P + N + bs - 1) // bs
    nb = R * blocks_per_req * 2 + 64
    root = args.root
    shutil.rmtree(root, ignore_errors=True)
    mounts = [os.path.join(root, f"nvme{d}") for d in range(args.drives)]
    nchunks = R * (P // g.chunk_tokens)
    spf = max(16, (nchunks + args.drives - 1) // args.drives)
    store = TuttiKVStore(root, g, capacity_chunks=spf * args.drives, mounts=mounts, device=args.device,
                         segment_file_slots=spf, namespace=b"ttft",
                         runtime_options={"controller_threads": args.controller_threads, "leases": 128,
                                          "max_ctas_per_op": args.ctas_per_layer, "slots_per_lease": 16,
                                          "queue_depth": 1024, "emulator_media": args.media,
                                          "image_budget_bytes": spf * (g.chunk_bytes + (128 << 10)) + (128 << 20),
                                          "async_completion": bool(args.async_completion)})
    store.open()
    model = LlamaModel(cfg, dev)
    pool = torch.zeros(g.pool_shape(nb), dtype=g.dtype, device=dev)
    engine = KVEngine(store, g, device=dev)
    engine.bind(pool)
    rng = np.random.default_rng(0)
    prompts = [torch.from_numpy(rng.integers(0, cfg.vocab, size=P + N)) for _ in range(R)]
    dev_prompts = [p.to(dev) for p in prompts]
    # Persist each request's prefix (its KV from a real prefill of the prefix).
    setup_tables = [torch.arange(r * blocks_per_req, (r + 1) * blocks_per_req) for r in range(R)]
    for r in range(R):
        model.prefill([prompts[r][:P]], [0], [setup_tables[r]], pool)
        keys = chunk_keys_for_tokens(prompts[r][:P].tolist(), g.chunk_tokens)
        comp = engine.store_chunks(keys, setup_tables[r][: P // bs])
        comp.wait()
    engine.wait_idle()
    torch.cuda.synchronize()

    def one(mode: str, it: int) -> float:
        # fresh, randomly placed blocks for every iteration
        perm = torch.from_numpy(np.random.default_rng(100 + it).permutation(nb)[: R * blocks_per_req])
        tables = [perm[r * blocks_per_req:(r + 1) * blocks_per_req] for r in range(R)]
        # block tables on the device before the clock starts (a serving engine keeps them
        # there); no host-to-device copy is then queued behind the layer waits of the prefill
        dev_tables = [t.to(dev) for t in tables]
        pool.zero_()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        if mode == "recompute":
            for r in range(R):
                model.prefill([dev_prompts[r]], [0], [dev_tables[r]], pool)
        else:
            keys, hit = [], []
            for r in range(R):
                k = chunk_keys_for_tokens(prompts[r][:P].tolist(), g.chunk_tokens)
                hit.append(engine.lookup_prefix_keys(k))
                keys.extend(k[: hit[-1] // g.chunk_tokens])
            table = torch.cat([tables[r][: hit[r] // bs] for r in range(R)])
            new = [dev_prompts[r][hit[r]:] for r in range(R)]
            if mode == "layerwise":
                plan = engine.start_read_plan(keys, table, window=args.window)
                model.prefill(new, hit, dev_tables, pool, wait_layer=plan.wait_layer)
                e.record()
                plan.finish()
            else:
                comp = engine.load(keys, table)
                comp.wait()
                torch.cuda.current_stream().wait_stream(engine.io_stream)
                model.prefill(new, hit, dev_tables, pool)
        if mode == "recompute" or mode == "restore_then_prefill":
            e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e)

    def checked(mode: str, it: int) -> float:
        try:
            return one(mode, it)
        except Exception:
            # the drives' counters say whether a restore waited on the media, the copies or the queues
            print(json.dumps({"failed_in": mode, "controllers": store.runtime.controller_stats()}), file=sys.stderr)
            raise

    # Shape warm-up: one prefill of the timed shapes before any restore runs.
    # Its first GEMMs of a new shape make cuBLAS load kernels, and a kernel
    # load takes a context-wide lock until the running kernels finish; with a
    # restore in flight that is the io kernel, which waits for the drives, whose
    # copies wait for the lock (measured: a 10 s stall of the first layerwise
    # restore). A serving engine does the same in its warm-up / graph capture.
    hit0 = [P] * R
    warm_tables = [torch.arange(r * blocks_per_req, (r + 1) * blocks_per_req).to(dev) for r in range(R)]
    model.prefill([dev_prompts[r][P:] for r in range(R)], hit0, warm_tables, pool)
    torch.cuda.synchronize()

    from ..common.clocks import ClockSampler

    out = {}
    for mode in args.modes:
        for w in range(args.warmup):
            checked(mode, 1000 + w)
        sampler = ClockSampler([args.device]).start()
        ts = [checked(mode, i) for i in range(args.iters)]
        out[mode] = {"p50_ms": round(statistics.median(ts), 2), "samples_ms": [round(t, 2) for t in ts],
                     "clocks": sampler.stop()}
    # correctness: logits from the layerwise path equal those of a full recompute
    store.close()
    shutil.rmtree(root, ignore_errors=True)
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--requests", type=int, default=8)
    p.add_argument("--prefix", type=int, default=32768)
    p.add_argument("--new", type=int, default=512)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--drives", type=int, default=4)
    p.add_argument("--controller-threads", type=int, default=1)
    p.add_argument("--media", choices=["memory", "files"], default="memory")
    p.add_argument("--reference", action="store_true",
                   help="also time the reference's staged restore (baseline/_ref) on the same workload")
    p.add_argument("--ctas-per-layer", type=int, default=32)
    p.add_argument("--window", type=int, default=4)
    p.add_argument("--async-completion", action="store_true",
                   help="split submit/drain launches: each layer's drain runs on the compute stream")
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--device", type=int, default=0)
    p.add_argument("--modes", nargs="+", default=["layerwise", "restore_then_prefill", "recompute"])
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_ttft"))
    args = p.parse_args(argv)
    t0 = time.time()
    res = run(args)
    if args.reference:
        import subprocess

        torch.cuda.empty_cache()  # the reference run allocates its own pool and model
        cmd = [sys.executable, "-m", "tutti_b200.benchmarks.ttft_reference", "--requests", str(args.requests),
               "--prefix", str(args.prefix), "--new", str(args.new), "--layers", str(args.layers),
               "--iters", str(args.iters), "--warmup", str(args.warmup), "--device", str(args.device)]
        out = subprocess.run(cmd, capture_output=True, text=True)
        lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
        res["reference"] = json.loads(lines[-1]) if lines else {"error": (out.stderr or out.stdout)[-400:]}
    line = {"metric": "ttft_p50_ms", "value": res.get("layerwise", {}).get("p50_ms"), "unit": "ms",
            "higher_is_better": False, "modes": res,
            "config": {"model": "llama-3.1-8b (random init)", "requests": args.requests, "prefix_tokens": args.prefix,
                       "new_tokens": args.new, "drives": args.drives, "media": args.media, "dtype": "bf16"},
            "wall_s": round(time.time() - t0, 1)}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
