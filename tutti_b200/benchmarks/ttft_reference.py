"""TTFT of the same long-prefix workload through the reference's own restore path.

    python -m tutti_b200.benchmarks.ttft_reference [--requests 8] [--prefix 32768] [--new 512]

The reference build (installed under baseline/_ref) restores each request's
cached prefix with its stock staged path: ``tutti.engine.core.KVEngine`` over
``tutti.storage.memory.MemoryKVStore`` (host DRAM), a pinned ``RingWindow``
staging bank and ``PagedTransferHooks`` scattering every layer into the paged
pool with the reference's K7 kernel (``tutti_kv_transfer``). The prefill is
this package's random-init Llama (the same model as ``benchmarks.ttft``), so
the two runs differ only in how the prefix KV reaches the pool. Two modes:

* ``reference_restore_then_prefill``: every layer restored and scattered, then
  the prefill of the new tokens;
* ``reference_layerwise``: the prefill's layer l waits (on the host) for layer
  l's restore and scatter; later layers keep reading meanwhile.

Runs in a process of its own: the reference's ``tutti`` package must win over
this repository's ``tutti`` import path.
"""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _reference_first() -> None:
    here = {ROOT, os.path.abspath(os.getcwd())}
    sys.path[:] = [REF_DIR] + [p for p in sys.path if os.path.abspath(p or ".") not in here] + [ROOT]
    for name in [m for m in sys.modules if m == "tutti" or m.startswith("tutti.")]:
        del sys.modules[name]


def main(argv=None) -> int:
    import argparse
    import json
    import statistics

    p = argparse.ArgumentParser()
    p.add_argument("--requests", type=int, default=8)
    p.add_argument("--prefix", type=int, default=32768)
    p.add_argument("--new", type=int, default=512)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--device", type=int, default=0)
    args = p.parse_args(argv)
    if not os.path.isdir(os.path.join(REF_DIR, "tutti")):
        print(json.dumps({"unavailable": "reference package not installed under baseline/_ref"}))
        return 0
    _reference_first()
    import numpy as np
    import torch

    from tutti.engine.core import KVEngine
    from tutti.engine.staging import RingWindow
    from tutti.integration.vllm.worker import PagedTransferHooks
    from tutti.storage.memory import MemoryKVStore
    from tutti_kv_transfer import discover_engine_format

    from tutti_b200.models.llama import LLAMA_3_1_8B, LlamaConfig, LlamaModel

    dev = torch.device("cuda", args.device)
    torch.cuda.set_device(dev)
    cfg = LLAMA_3_1_8B if args.layers == 32 else LlamaConfig(layers=args.layers)
    g = cfg.geometry()
    R, P, N = args.requests, args.prefix, args.new
    bs, CT, L = g.block_size, g.chunk_tokens, cfg.layers
    bpc = CT // bs
    blocks_per_req = (P + N + bs - 1) // bs
    nb = R * blocks_per_req * 2 + 64
    seg = g.segment_bytes
    model = LlamaModel(cfg, dev)
    pool = torch.zeros(g.pool_shape(nb), dtype=g.dtype, device=dev)
    chunks_per_req = P // CT
    store = MemoryKVStore(seg, R * chunks_per_req + 16)
    wave = R * chunks_per_req
    engine = KVEngine({"chunk_tokens": CT, "chunk_kv_bytes": seg * L, "max_chunks_per_wave": wave,
                       "num_layers": L}, store)
    bank = 2 * wave
    staging = torch.empty(2 * bank * seg, dtype=torch.uint8, pin_memory=True)
    raw = staging.numpy()
    read_window = RingWindow(raw, bank, seg, capacity_per_wave=wave, slot_base=0)
    write_window = RingWindow(raw, bank, seg, capacity_per_wave=wave, slot_base=bank)
    fmt = discover_engine_format(pool[0], use_mla=False)
    hooks = PagedTransferHooks(lambda i: pool[i], staging, seg, CT, bs, fmt)
    engine.bind({}, read_window, L, bpc, write_window=write_window, gather_fn=hooks.gather,
                scatter_fn=hooks.scatter, force_staged=True)

    rng = np.random.default_rng(0)
    prompts = [torch.from_numpy(rng.integers(0, cfg.vocab, size=P + N)) for _ in range(R)]
    setup_tables = [torch.arange(r * blocks_per_req, (r + 1) * blocks_per_req) for r in range(R)]
    all_keys, src_tables = [], []
    for r in range(R):
        model.prefill([prompts[r][:P]], [0], [setup_tables[r]], pool)
        keys, _ = engine.hash_keys(prompts[r][:P].tolist())
        all_keys.extend(keys)
        src_tables.extend(setup_tables[r][c * bpc:(c + 1) * bpc].tolist() for c in range(chunks_per_req))
    torch.cuda.synchronize()
    if engine.plan_store(all_keys) is None:
        print(json.dumps({"unavailable": "reference plan_store refused the prefixes"}))
        return 0
    for layer in range(L):
        engine.store_layer(all_keys, layer, src_tables)
    engine.wait_idle()
    engine.confirm_store(all_keys)

    def one(mode: str, it: int) -> float:
        perm = torch.from_numpy(np.random.default_rng(100 + it).permutation(nb)[: R * blocks_per_req])
        tables = [perm[r * blocks_per_req:(r + 1) * blocks_per_req] for r in range(R)]
        pool.zero_()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        keys, hit = [], []
        for r in range(R):
            k, _ = engine.hash_keys(prompts[r][:P].tolist())
            hit.append(engine.lookup_prefix_keys(k))
            keys.extend(k[: hit[-1] // CT])
        dst = []
        for r in range(R):
            t = tables[r].tolist()
            dst.extend(t[c * bpc:(c + 1) * bpc] for c in range(hit[r] // CT))
        new = [prompts[r][hit[r]:] for r in range(R)]
        handles = [engine.load_layer(keys, layer, dst) for layer in range(L)]
        if mode == "reference_layerwise":
            model.prefill(new, hit, tables, pool, wait_layer=lambda layer: handles[layer].wait())
        else:
            for h in handles:
                h.wait()
            model.prefill(new, hit, tables, pool)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e)

    out = {}
    for mode in ("reference_restore_then_prefill", "reference_layerwise"):
        for w in range(args.warmup):
            one(mode, 1000 + w)
        ts = [one(mode, i) for i in range(args.iters)]
        out[mode] = {"p50_ms": round(statistics.median(ts), 2), "samples_ms": [round(t, 2) for t in ts]}
    engine.close()
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
