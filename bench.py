#!/usr/bin/env python
"""Headline benchmark: SSD->HBM KV restore GB/s (whole job, all ranks).

One step restores one 32,768-token Llama-3.1-8B KV prefix (32 layers x 8 KV
heads x 128 dims, bf16, block 16: 2,048 blocks x 64 KiB x 32 layers = 4.29 GB)
from the segment-file store into seeded random blocks of a 16,384-block paged
pool in HBM, through the public API (TuttiKVStore.get_paged -> StorageRuntime
submit -> fused sm_100a NVMe io kernel -> emulated NVMe controllers serving the
segment files from the host's page cache). Each rank restores its own prefix
(weak scaling). Device time is measured with CUDA events on the launching
stream, max over ranks. Inputs (4.29 GB per step) are far larger than L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--drives D]
    python bench.py --impl reference     # the reference's own build
    python bench.py --impl posix         # CPU-initiated pread + cudaMemcpy baseline

For N > 1 launch with torch.distributed.run (one rank per GPU).
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "kv_restore_GBps"
BASELINE_GBPS = None  # the reference publishes no B200 number for this config
ZERO_COPY_GBPS = 51.4  # GPU reads of pinned host memory, measured on this pool's B200s


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--no-numa-bind", action="store_true",
                   help="keep every CPU (default: each rank runs on its GPU's NUMA node)")
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="tutti", choices=["tutti", "reference", "posix"])
    p.add_argument("--drives", type=int, default=4, help="emulated NVMe drives (striped mounts) per rank")
    p.add_argument("--prefix-tokens", type=int, default=32768)
    p.add_argument("--pool-blocks", type=int, default=16384)
    p.add_argument("--root", default=os.environ.get("TUTTI_BENCH_ROOT", "/tmp/tutti_bench"))
    p.add_argument("--controller-threads", type=int, default=0, help="0: auto")
    p.add_argument("--direct-io", action="store_true", help="O_DIRECT backing reads (drive-bound)")
    p.add_argument("--no-verify", action="store_true")
    p.add_argument("--timing", action="store_true", help="per-command %%globaltimer breakdown (stderr)")
    p.add_argument("--leases", type=int, default=192, help="queue leases (CTAs) per GPU")
    p.add_argument("--ctas", type=int, default=0, help="CTAs one restore may use (0: by media)")
    p.add_argument("--slots", type=int, default=16)
    p.add_argument("--media", choices=["memory", "files"], default="memory",
                   help="emulated drive media: in-memory image DMA'd into HBM, or the files (pread)")
    p.add_argument("--drive-gbps", type=float, default=0.0, help="per-drive transfer cap (0: none)")
    p.add_argument("--e2e-parts", default="h2d,readback", help=argparse.SUPPRESS)  # diagnostics
    p.add_argument("--async-completion", action="store_true",
                   help="split submit/drain: the drain starts once the drives have posted every CQE")
    p.add_argument("--inflight", type=int, default=2, help="restores submitted ahead")
    p.add_argument("--direct-reads", action="store_true",
                   help="drives DMA each read straight into the pool pages (no staging, no movers)")
    p.add_argument("--provider", choices=["emulated", "snvme_fake"], default="emulated",
                   help="controller provider: emulated drives, or the snvme client over a fake driver")
    p.add_argument("--emulator-skip-data", action="store_true", help="diagnostic: controllers move no data")
    p.add_argument("--staging-wc", action="store_true", help="write-combined staging slots")
    p.add_argument("--idle-spins", type=int, default=0,
                   help="queue scans before an idle emulated-drive worker sleeps (0: auto)")
    p.add_argument("--emulator-reads", choices=["mmap", "pread"], default="pread",
                   help="how the emulated drives read page-cached segment files")
    return p.parse_args()


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons every 100 ms during the timed region.

    (The same sampler as tutti_b200.common.clocks, kept here so that the reference arm
    imports nothing of this package.)
    """

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.rows = []
        self._proc = None
        self._t = None

    def start(self):
        if shutil.which("nvidia-smi") is None:
            return self
        # one long-running sampler (-lms) instead of a process per sample
        self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)

        def run():
            for line in self._proc.stdout:
                f = [x.strip() for x in line.split(",")]
                try:
                    if len(f) >= 8 and int(f[0]) in self.gpus:
                        self.rows.append(f)
                except ValueError:
                    continue

        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        time.sleep(0.3)  # first sample before the timed region starts
        return self

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._t:
            self._t.join(timeout=5)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


NUMA_BIND: dict = {"bound": False, "why": "not requested"}


def numa_bind(local: int) -> dict:
    """Run this rank's host work on its GPU's NUMA node (both arms; the harness, not either product).

    The calling thread, and every thread it starts afterwards (drive threads,
    staging copies), is restricted to the CPUs sysfs lists as local to the
    GPU's PCIe function, so page-locked buffers allocated afterwards land on
    that node. Nothing outside this process changes.
    """
    import torch

    try:
        p = torch.cuda.get_device_properties(local)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bdf}/local_cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                a, _, b = part.partition("-")
                if a:
                    cpus.update(range(int(a), int(b or a) + 1))
    except (OSError, ValueError, RuntimeError, AttributeError) as e:
        return {"bound": False, "why": f"{type(e).__name__}: {e}"[:120]}
    allowed = cpus & os.sched_getaffinity(0)
    if not allowed:
        return {"bound": False, "gpu": bdf, "why": "no local CPU is allowed"}
    os.sched_setaffinity(0, allowed)
    return {"bound": True, "gpu": bdf, "cpus": len(allowed)}


def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    global NUMA_BIND
    torch.cuda.set_device(local)  # before the first CUDA query: no context on another GPU
    if os.environ.get("TUTTI_BENCH_NUMA_BIND", "1") != "0":
        NUMA_BIND = numa_bind(local)
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(world, value: float) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(world, value: float) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_STAGED_NOTE = ("reference staged restore: KVEngine over MemoryKVStore (host DRAM) + RingWindow pinned "
                   "staging + PagedTransferHooks -> tutti_kv_transfer single_layer_kv_transfer (K7); the "
                   "reference's snvme SSD path needs drives and a kernel module this pool lacks")


def _ensure_reference_kernels() -> str | None:
    """Build the reference's own ``tutti_kv_transfer`` extension into baseline/_ref if it is missing.

    The sources are the reference's ``csrc/kv_transfer`` tree, built unmodified by
    its own setup.py with the arch list set for sm_100a. Returns a reason string
    when the extension cannot be had.
    """
    import glob

    if glob.glob(os.path.join(REF_DIR, "tutti_kv_transfer", "_native*.so")):
        return None
    # the reference checkout next to this repository, unless named
    src = os.environ.get("TUTTI_REFERENCE_SRC") or os.path.join(os.path.dirname(ROOT), "reference")
    if not os.path.isdir(os.path.join(src, "csrc", "kv_transfer")):
        return "reference kv_transfer extension not built and its sources are not on this machine"
    import tempfile

    tmp = tempfile.mkdtemp(prefix="refkvt_")
    shutil.copytree(os.path.join(src, "csrc", "kv_transfer"), os.path.join(tmp, "csrc", "kv_transfer"))
    shutil.copy(os.path.join(src, "VERSION"), os.path.join(tmp, "VERSION"))
    env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a", MAX_JOBS="8")
    r = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                        "--find-links", "/opt/wheelhouse", "--target", REF_DIR,
                        os.path.join(tmp, "csrc", "kv_transfer")], env=env, capture_output=True, text=True)
    shutil.rmtree(tmp, ignore_errors=True)
    if r.returncode != 0:
        return "building the reference kv_transfer extension failed: " + (r.stderr or r.stdout)[-200:].replace("\n", " ")
    return None


def reference_arm(args):
    """The reference's own build on the same config: its stock staged restore.

    Path (all reference code, imported from baseline/_ref, nothing of this
    repository): ``tutti.engine.core.KVEngine`` over ``tutti.storage.memory.MemoryKVStore``
    (the prefix in host DRAM), staged through a pinned ``RingWindow`` and scattered
    into the paged pool by ``PagedTransferHooks`` (tutti/integration/vllm/worker.py:256-460)
    with the reference's K7 kernel (csrc/kv_transfer/src/mem_kernels.cu:66-130).
    One step restores the 32 layers of the prefix with ``load_layer`` per layer
    (tutti/engine/core.py:1936) and waits for every layer's scatter.
    """
    rank = int(os.environ.get("RANK", "0"))

    def unavailable(reason: str) -> int:
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": reason}))
        return 0

    if not os.path.isdir(os.path.join(REF_DIR, "tutti")):
        return unavailable("reference package not installed under baseline/_ref")
    why = _ensure_reference_kernels()
    if why:
        return unavailable(why)
    # The reference's packages must win over this repository's `tutti` import path.
    here = {ROOT, os.path.abspath(os.getcwd())}
    sys.path[:] = [REF_DIR] + [p for p in sys.path if os.path.abspath(p or ".") not in here]
    for name in [m for m in sys.modules if m == "tutti" or m.startswith("tutti.")]:
        del sys.modules[name]
    import numpy as np
    import torch

    try:
        import tutti
        from tutti.engine.core import KVEngine
        from tutti.engine.staging import RingWindow
        from tutti.integration.vllm.worker import PagedTransferHooks
        from tutti.storage.memory import MemoryKVStore
        from tutti_kv_transfer import discover_engine_format
    except Exception as e:  # noqa: BLE001 - one line for the driver
        return unavailable(f"reference import failed: {type(e).__name__}: {e}")
    if not os.path.abspath(tutti.__file__).startswith(REF_DIR) or "tutti_b200" in sys.modules:
        return unavailable("reference import resolved outside baseline/_ref")
    if not torch.cuda.is_available():
        return unavailable("no CUDA device on this machine (the reference's K7 scatter needs one)")

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    L, H, D, BS, CT = 32, 8, 128, 16, 256  # Llama-3.1-8B KV, block 16, 256-token chunks
    nblk = args.prefix_tokens // BS
    nchunks = args.prefix_tokens // CT
    bpc = CT // BS
    seg = CT * 2 * H * D * 2  # one layer of one chunk: K and V rows, bf16
    layers = [torch.empty((2, args.pool_blocks, BS, H, D), dtype=torch.bfloat16, device=dev) for _ in range(L)]
    store = MemoryKVStore(seg, nchunks + 16)
    engine = KVEngine({"chunk_tokens": CT, "chunk_kv_bytes": seg * L, "max_chunks_per_wave": nchunks,
                       "num_layers": L}, store)
    # The worker's staged binding (worker.py:2320-2390): two banks of lookahead_k (2) layers each.
    bank = 2 * nchunks
    staging = torch.empty(2 * bank * seg, dtype=torch.uint8, pin_memory=True)
    raw = staging.numpy()
    read_window = RingWindow(raw, bank, seg, capacity_per_wave=nchunks, slot_base=0)
    write_window = RingWindow(raw, bank, seg, capacity_per_wave=nchunks, slot_base=bank)
    fmt = discover_engine_format(layers[0], use_mla=False)
    hooks = PagedTransferHooks(lambda i: layers[i], staging, seg, CT, BS, fmt)
    engine.bind({}, read_window, L, bpc, write_window=write_window, gather_fn=hooks.gather,
                scatter_fn=hooks.scatter, force_staged=True)

    rng = np.random.default_rng(rank)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    src_blocks = rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, bpc)
    src_idx = torch.from_numpy(src_blocks.reshape(-1)).to(dev)
    ref = torch.randn((L, 2, nblk, BS, H, D), dtype=torch.bfloat16, device=dev, generator=gen)
    for i in range(L):
        layers[i][:, src_idx] = ref[i]
    tokens = torch.randint(0, 128_000, (args.prefix_tokens,), generator=torch.Generator().manual_seed(7 + rank))
    keys, _ = engine.hash_keys(tokens.tolist())
    t0 = time.perf_counter()
    plan = engine.plan_store(keys)
    if plan is None:
        return unavailable("reference plan_store refused the prefix")
    for i in range(L):
        engine.store_layer(keys, i, [list(map(int, b)) for b in src_blocks])
    engine.wait_idle()
    engine.confirm_store(keys)
    store_s = time.perf_counter() - t0
    bytes_per_step = nblk * L * 2 * BS * H * D * 2

    perms = [rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, bpc)
             for _ in range(args.warmup + args.steps)]
    tables = [[list(map(int, b)) for b in p] for p in perms]
    pinned_tables = [torch.from_numpy(p.reshape(-1).copy()).pin_memory() for p in perms]
    dev_table = torch.empty(nblk, dtype=torch.int64, device=dev)
    checksum = torch.zeros(1, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    launches = [0]

    def run_steps(first: int, count: int, e2e: bool) -> None:
        for i in range(first, first + count):
            if e2e:
                dev_table.copy_(pinned_tables[i], non_blocking=True)
            handles = [engine.load_layer(keys, layer, tables[i]) for layer in range(L)]
            for h in handles:
                h.wait()
            launches[0] += L  # one K7 scatter launch per layer (the whole prefix is one wave)
            if e2e:
                checksum.copy_(layers[0][0, int(perms[i].reshape(-1)[0])].float().sum().reshape(1),
                               non_blocking=True)
        stream.synchronize()

    run_steps(0, args.warmup, False)
    barrier(world)
    sampler = ClockSampler(list(range(world))).start() if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    ev0.record(stream)
    launches[0] = 0
    run_steps(args.warmup, args.steps, False)
    ev1.record(stream)
    torch.cuda.synchronize()
    dev_ms = ev0.elapsed_time(ev1) / args.steps
    n_launch = launches[0]
    barrier(world)
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    run_steps(args.warmup, args.steps, True)
    ev3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev2.elapsed_time(ev3) / args.steps
    barrier(world)
    clocks = sampler.stop() if sampler else None
    last = torch.from_numpy(perms[-1].reshape(-1)).to(dev)
    ok = all(bool(torch.equal(layers[i][:, last], ref[i])) for i in range(L))
    ok_all = max_over_ranks(world, 0.0 if ok else 1.0) == 0.0
    ms = max_over_ranks(world, dev_ms)
    e2e = max_over_ranks(world, e2e_ms)
    total_bytes = sum_over_ranks(world, float(bytes_per_step))
    engine.close()
    if rank == 0:
        value = total_bytes / (ms / 1e3) / 1e9
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (randn KV of the named shape; prefix held by the reference's MemoryKVStore)",
            "config": {"model": "llama-3.1-8b KV (32L x 8H x 128D, block 16)", "global_batch": world, "numa_bind": NUMA_BIND,
                       "seq_len": args.prefix_tokens, "parallelism": f"dp{world} (one prefix per rank)",
                       "pool_blocks": args.pool_blocks, "path": REF_STAGED_NOTE,
                       "l2": "inputs (4.29 GB/step) larger than L2"},
            "e2e": {"value": round(total_bytes / (e2e / 1e3) / 1e9, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": nblk * 8, "d2h_bytes_per_step": 4},
            "gpu_launches": n_launch, "verified": ok_all, "store_setup_s": round(store_s, 2), "clocks": clocks,
        }))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0 if ok_all else 1


def measure_drive_gbps(store, keys, threads_per_drive: int, piece: int = 1 << 20, repeats: int = 2) -> float:
    """Host-only read of the prefix's segment-file bytes, split like the emulated drives split it.

    The same files, byte ranges, 1 MiB pieces and threads per drive as the
    emulated controllers, read with ``preadv`` into per-thread buffers and no
    GPU involved: the ceiling of the drives this bench emulates (their PRP walk
    and the writes into mapped staging slots come on top).
    """
    import concurrent.futures as cf

    n = len(store.mounts)
    span = store.geometry.num_layers * store.stored["segment_bytes"]
    per_drive: dict[int, list] = {}
    for k in keys:
        uri, off, slot, _gen = store.objects.lookup(bytes(k))
        per_drive.setdefault(slot % n, []).append((uri[len("file://"):], off))
    jobs, total = [], 0
    for items in per_drive.values():
        pieces = [(p, o + b, min(piece, span - b)) for p, o in items for b in range(0, span, piece)]
        total += sum(x[2] for x in pieces)
        jobs += [pieces[t::threads_per_drive] for t in range(threads_per_drive)]
    fds = {p: os.open(p, os.O_RDONLY) for p in {x[0] for j in jobs for x in j}}

    def work(pieces):
        buf = memoryview(bytearray(8 * piece))  # 8 slots per thread, as a lease's staging slots
        for i, (p, o, ln) in enumerate(pieces):
            at = (i % 8) * piece
            os.preadv(fds[p], [buf[at:at + ln]], o)

    best = 0.0
    try:
        with cf.ThreadPoolExecutor(len(jobs)) as ex:
            for _ in range(repeats):
                t0 = time.perf_counter()
                list(ex.map(work, jobs))
                best = max(best, total / (time.perf_counter() - t0) / 1e9)
    finally:
        for fd in fds.values():
            os.close(fd)
    return best


def measure_dma_gbps(dev, piece: int = 1 << 20, total: int = 2 << 30) -> float:
    """Copy-engine rate of the drives' transfers: 1 MiB copies from page-locked host memory into HBM.

    The same transfer size and direction the emulated drives issue for each
    READ command, back to back on one stream, timed with CUDA events.
    """
    import torch

    src = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dst = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream(dev)
    n = total // piece
    k = (256 << 20) // piece
    with torch.cuda.stream(s):
        for i in range(k):  # warm-up
            dst[i * piece:(i + 1) * piece].copy_(src[i * piece:(i + 1) * piece], non_blocking=True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(n):
            j = i % k
            dst[j * piece:(j + 1) * piece].copy_(src[j * piece:(j + 1) * piece], non_blocking=True)
        e1.record(s)
    e1.synchronize()
    return total / (e0.elapsed_time(e1) / 1e3) / 1e9


def main():
    args = parse()
    if args.no_numa_bind:
        os.environ["TUTTI_BENCH_NUMA_BIND"] = "0"
    # More hardware queues (before CUDA starts): the emulated drives' copy
    # streams then rarely share one with a stream that has work waiting on an
    # io kernel.
    os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
    # Load every kernel when CUDA starts: loading one lazily while an io kernel
    # waits for the drives takes a context-wide lock that also stalls the
    # drives' copy calls until the io kernel's deadline.
    os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")
    if args.impl == "reference":
        return reference_arm(args)
    import numpy as np
    import torch

    from tutti_b200.models.kv_geometry import LLAMA3_8B
    from tutti_b200.storage.tutti_store import TuttiKVStore
    from tutti_b200.index.chunk_index import chunk_keys_for_tokens

    world, rank, local = dist_setup()
    g = LLAMA3_8B
    dev = torch.device("cuda", local)
    nblk = args.prefix_tokens // g.block_size
    nchunks = args.prefix_tokens // g.chunk_tokens
    root = os.path.join(args.root, f"r{rank}")
    shutil.rmtree(root, ignore_errors=True)
    mounts = [os.path.join(root, f"nvme{d}") for d in range(args.drives)]
    ncpu = os.cpu_count() or 8
    # 3 workers per emulated drive measured best at 1 and 4 GPUs (16 and 32 host cores);
    # fewer when the box has under two cores per worker
    idle_spins = args.idle_spins or 2000  # 64 measured no different, even on 4 cores
    memory = args.media == "memory"
    if memory:
        # a drive worker only walks PRPs and issues copies: one per drive
        threads = args.controller_threads or 1
    else:
        threads = args.controller_threads or max(1, min(3, (2 * ncpu // max(1, world)) // max(1, args.drives)))
    ctas = args.ctas or (32 if memory else 96)
    opts = {"controller_threads": threads, "direct_io": bool(args.direct_io), "leases": args.leases,
            "emulator_media": args.media, "drive_gbps": args.drive_gbps,
            "async_completion": bool(args.async_completion), "async_fallback_us": 500000, "queue_depth": 1024,
            "max_ctas_per_op": ctas, "slots_per_lease": args.slots, "slot_bytes": 1 << 20, "mdts_bytes": 1 << 20, "timing": bool(args.timing),
            "emulator_skip_data": bool(args.emulator_skip_data), "emulator_reads": args.emulator_reads,
            "staging_write_combined": bool(args.staging_wc), "emulator_idle_spins": idle_spins,
            "direct_reads": bool(args.direct_reads), "nvme_provider": args.provider}
    backend = "nvme-gpu" if args.impl == "tutti" else "posix"
    if backend == "posix":
        opts = {"threads": max(4, ncpu // max(1, world)), "direct_io": bool(args.direct_io)}
    # capacity: the prefix plus one spare file group
    spf = max(16, (nchunks + args.drives - 1) // args.drives)
    if memory:  # each drive's image arena holds its segment file (allocated when the drive is created)
        opts["image_budget_bytes"] = spf * (g.chunk_bytes + (128 << 10)) + (128 << 20)
    store = TuttiKVStore(root, g, capacity_chunks=spf * args.drives, mounts=mounts, device=local,
                         backend=backend, runtime_options=opts, segment_file_slots=spf,
                         namespace=b"bench")
    store.open()
    pool = torch.empty(g.pool_shape(args.pool_blocks), dtype=g.dtype, device=dev)
    store.register_pool(pool)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    # Source prefix in the pool at seeded random blocks, persisted once (untimed setup).
    rng = np.random.default_rng(rank)
    src_blocks = rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, g.blocks_per_chunk)
    src_idx = torch.from_numpy(src_blocks.reshape(-1)).to(dev)
    ref = torch.randn((g.num_layers, g.planes, nblk, g.block_size, g.heads_per_rank, g.head_dim), dtype=g.dtype,
                      device=dev, generator=gen)
    pool[:, :, src_idx] = ref
    tokens = torch.randint(0, 128_000, (args.prefix_tokens,), generator=torch.Generator().manual_seed(7 + rank))
    keys = chunk_keys_for_tokens(tokens.tolist(), g.chunk_tokens)
    t0 = time.perf_counter()
    try:
        store.put_paged(keys, src_blocks).wait()
    except Exception:
        print(json.dumps({"controllers": store.runtime.controller_stats()}), file=sys.stderr)
        raise
    store_s = time.perf_counter() - t0
    store.warm_targets()
    bytes_per_step = nblk * g.num_layers * g.block_layer_bytes
    # roofline: the emulated drives' own ceiling, all ranks at once
    barrier(world)
    if backend != "nvme-gpu":
        drive_gbps = 0.0
    elif memory:
        drive_gbps = measure_dma_gbps(dev)  # the copies the drives issue, with no protocol around them
    else:
        drive_gbps = measure_drive_gbps(store, keys, threads)  # host-only reads of the files
    drive_total = sum_over_ranks(world, drive_gbps)
    if args.drive_gbps:
        drive_total = min(drive_total, args.drive_gbps * args.drives * world)

    perms = [rng.permutation(args.pool_blocks)[:nblk].reshape(nchunks, g.blocks_per_chunk)
             for _ in range(args.warmup + args.steps)]
    pinned_tables = [torch.from_numpy(p.reshape(-1).copy()).pin_memory() for p in perms]
    dev_table = torch.empty(nblk, dtype=torch.int64, device=dev)
    checksum = torch.zeros(1, dtype=torch.float32).pin_memory()
    # The restores run on an io stream of their own and the per-step input and
    # result copies on a copy stream (as a serving engine keeps them), so no
    # copy is ever queued behind a running io kernel.
    stream = torch.cuda.Stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    launches = [0]
    io_bytes = [0, 0]  # per e2e run: H2D command arenas, D2H statuses

    parts = set(args.e2e_parts.split(","))

    def result_readback(j: int) -> None:
        if "readback" not in parts:
            return
        with torch.cuda.stream(copy_stream):  # D2H: the step's result (a checksum of its first restored block)
            if "nosum" in parts:
                checksum.view(torch.bfloat16)[:2].copy_(pool[0, 0, int(perms[j].reshape(-1)[0]), 0, 0, :2],
                                                        non_blocking=True)
            else:
                checksum.copy_(pool[0, 0, int(perms[j].reshape(-1)[0])].float().sum().reshape(1), non_blocking=True)

    def run_steps(first: int, count: int, e2e: bool) -> None:
        """``count`` restores with up to ``args.inflight`` submitted ahead (host work overlaps IO)."""
        pending = []
        for i in range(first, first + count):
            if e2e and "h2d" in parts:
                with torch.cuda.stream(copy_stream):  # H2D: this step's block table
                    dev_table.copy_(pinned_tables[i], non_blocking=True)
                stream.wait_stream(copy_stream)
            comp = store.get_paged(keys, perms[i], stream=stream)
            launches[0] += len(comp._ios)
            if e2e and backend == "nvme-gpu":
                prof = store.runtime.last_submit_profile()  # the command arena this step copied, and back
                io_bytes[0] += prof.get("h2d_bytes", 0)
                io_bytes[1] += prof.get("d2h_bytes", 0)
            pending.append((i, comp))
            while len(pending) >= args.inflight:
                j, c = pending.pop(0)
                c.wait()
                if e2e:
                    result_readback(j)
        for j, c in pending:
            c.wait()
            if e2e:
                result_readback(j)
        stream.synchronize()
        copy_stream.synchronize()

    run_steps_plain = run_steps

    def checked(first: int, count: int, e2e: bool) -> None:
        try:
            run_steps_plain(first, count, e2e)
        except Exception:
            print(json.dumps({"failed_in": "e2e" if e2e else "device-timed",
                              "controllers": store.runtime.controller_stats()}), file=sys.stderr)
            raise

    run_steps = checked  # noqa: F811 - failures report the drives' counters
    run_steps(0, args.warmup, False)
    barrier(world)
    sampler = ClockSampler(list(range(world))).start() if rank == 0 else None  # every GPU of the job
    # device-timed: K restores back to back
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    ev0.record(stream)
    launches[0] = 0
    run_steps(args.warmup, args.steps, False)
    ev1.record(stream)
    torch.cuda.synchronize()
    dev_ms = ev0.elapsed_time(ev1) / args.steps
    n_launch = launches[0]
    barrier(world)
    # end to end: + H2D block table from pinned memory + D2H result readback every step
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    run_steps(args.warmup, args.steps, True)
    ev3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev2.elapsed_time(ev3) / args.steps
    barrier(world)
    clocks = sampler.stop() if sampler else None

    ok = True
    if not args.no_verify:
        last = torch.from_numpy(perms[-1].reshape(-1)).to(dev)
        ok = bool(torch.equal(pool[:, :, last], ref))
    ok_all = max_over_ranks(world, 0.0 if ok else 1.0) == 0.0
    ms = max_over_ranks(world, dev_ms)
    e2e = max_over_ranks(world, e2e_ms)
    total_bytes = sum_over_ranks(world, float(bytes_per_step))
    timing = store.runtime.io_timing() if store.runtime and args.timing else {}
    stats = store.runtime.controller_stats() if store.runtime else []
    staging_where = "hbm" if store.runtime and store.runtime.staging_on_device() else "host"
    if args.timing and rank == 0:
        print(json.dumps({"io_timing": timing, "controllers": stats}), file=sys.stderr)
    store.close()
    if rank == 0:
        value = total_bytes / (ms / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None if BASELINE_GBPS is None else round(value / BASELINE_GBPS, 3),
            "dtype": "bf16",
            "data": ("synthetic (randn KV of the named shape; emulated NVMe drives with in-memory media, "
                     "copy-engine DMA into HBM staging)" if memory else
                     "synthetic (randn KV of the named shape; emulated NVMe over page-cached segment files)"),
            "config": {"model": "llama-3.1-8b KV (32L x 8H x 128D, block 16)", "global_batch": world, "numa_bind": NUMA_BIND,
                       "seq_len": args.prefix_tokens, "parallelism": f"dp{world} (one prefix per rank)",
                       "pool_blocks": args.pool_blocks, "drives_per_rank": args.drives,
                       "backing": "O_DIRECT" if args.direct_io else "page cache", "media": args.media,
                       "staging": staging_where,
                       "drive_gbps_cap": args.drive_gbps or None, "ctas": ctas, "slots": args.slots,
                       "controller_threads": threads, "impl": args.impl, "inflight": args.inflight,
                       "async_completion": bool(args.async_completion),
                       "direct_reads": bool(args.direct_reads), "provider": args.provider,
                       "emulator_reads": args.emulator_reads, "staging_write_combined": bool(args.staging_wc),
                       "emulator_idle_spins": idle_spins,
                       "l2": "inputs (4.29 GB/step) larger than L2"},
            "e2e": {"value": round(total_bytes / (e2e / 1e3) / 1e9, 3), "unit": "GB/s",
                    # the block table (pinned) and the command arena the runtime copies to the
                    # device each step; back: the result checksum and the per-command statuses
                    "h2d_bytes_per_step": nblk * 8 + io_bytes[0] // args.steps,
                    "d2h_bytes_per_step": 4 + io_bytes[1] // args.steps},
            "gpu_launches": n_launch,
            # Roofline: the drives' transfers. Memory media: the copy engines' rate for the
            # 1 MiB host->HBM copies every READ is served with (measured in this run, before
            # warm-up, no protocol around it), times the ranks; capped by --drive-gbps x drives.
            # File media: the GPU's zero-copy read of the host staging slots (51.4 GB/s on this
            # pool) against the host-only read rate of the files by the same threads.
            "roofline": ({"term": "copy-engine DMA of 1 MiB commands, page-locked host image -> HBM",
                          "per_gpu_gbps": round(drive_gbps, 3), "bound_gbps": round(drive_total, 3),
                          "fraction_of_bound": round(value / drive_total, 3) if drive_total else None}
                         if memory else
                         {"term": "PCIe zero-copy read of staging slots", "per_gpu_gbps": ZERO_COPY_GBPS,
                          "per_gpu_fraction": round(value / world / ZERO_COPY_GBPS, 3),
                          "emulated_drive_gbps": round(drive_total, 3),
                          "bound_gbps": round(min(ZERO_COPY_GBPS * world, drive_total or 1e9), 3),
                          "fraction_of_bound": round(value / min(ZERO_COPY_GBPS * world, drive_total or 1e9), 3)}),
            "verified": ok_all,
            "store_setup_s": round(store_s, 2),
            "clocks": clocks,
        }
        print(json.dumps(out))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    shutil.rmtree(root, ignore_errors=True)
    return 0 if ok_all else 1


if __name__ == "__main__":
    sys.exit(main())
