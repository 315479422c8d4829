"""Pure-host parts of the benchmark drivers: trace generation and the compute model."""
import argparse

from tutti_b200.benchmarks.serving_trace import FALLBACK_PEAKS, make_trace, prefill_seconds


def _args(**kw):
    base = dict(seed=0, distinct=512, zipf=1.1, min_prefix=8192, max_prefix=65536, length_scale=1.0,
                requests=400, reuse=0.8, warm=16)
    base.update(kw)
    return argparse.Namespace(**base)


def test_trace_is_seeded_and_shaped():
    a = make_trace(_args(), 256)
    assert a == make_trace(_args(), 256)
    assert all(r["tokens"] % 256 == 0 and 8192 - 256 <= r["tokens"] <= 65536 for r in a)
    reused = sum(r["prefix"] < 512 for r in a) / len(a)
    assert 0.7 < reused < 0.9
    # Zipf: the most popular prefix recurs
    counts = {}
    for r in a:
        counts[r["prefix"]] = counts.get(r["prefix"], 0) + 1
    assert max(counts.values()) >= 10
    # the same prefix id always has the same length
    lens = {}
    for r in a:
        assert lens.setdefault(r["prefix"], r["tokens"]) == r["tokens"]


def test_length_scale_shrinks_prefixes():
    a = make_trace(_args(length_scale=0.125), 256)
    assert all(256 <= r["tokens"] <= 8192 for r in a)


def test_prefill_model_grows_with_tokens_and_shrinks_with_tp():
    pk = dict(FALLBACK_PEAKS)
    assert prefill_seconds(0, 1000, 8, pk, 0.5) == 0.0
    one = prefill_seconds(4096, 0, 1, pk, 0.5)
    assert prefill_seconds(8192, 0, 1, pk, 0.5) > 2 * one * 0.99
    assert abs(prefill_seconds(4096, 0, 8, pk, 0.5) - one / 8) < 1e-12
    assert prefill_seconds(512, 32768, 1, pk, 0.5) < prefill_seconds(32768 + 512, 0, 1, pk, 0.5)


def test_io_sweep_shapes_cover_the_reference_batches():
    from tutti_b200.benchmarks.io_sweep import shape_for

    for target in (128, 486, 972, 1944, 3888):
        chunks, layers = shape_for(target)
        pages = chunks * 16 * layers
        assert layers <= 32 and abs(pages - target) / target < 0.02


def test_bench_reference_arm_prints_one_json_line():
    """The driver's reference arm contract: exactly one JSON line with impl=reference (no GPU needed)."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "1", "--steps", "2",
                          "--warmup", "3"], cwd=root, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference" and ("unavailable" in rec or "value" in rec)


def test_vllm_phase_runner_reaps_the_session_and_bounds_a_hang(tmp_path):
    """A phase that leaves a child holding its output, and one that hangs: neither blocks the harness."""
    import sys
    import time

    from tutti_b200.benchmarks.vllm_e2e import _run_phase_process

    # exits at once but leaves a grandchild (holding stdout) sleeping for a minute
    leaver = ("import subprocess, sys; subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(60)']);"
              " print('RESULT {}', flush=True)")
    t0 = time.monotonic()
    rc, out, err = _run_phase_process([sys.executable, "-c", leaver], None, 30, str(tmp_path), "leaver")
    assert rc == 0 and "RESULT {}" in out and time.monotonic() - t0 < 20
    # hangs: SIGUSR1 makes faulthandler dump the stacks, then the session is killed
    hang = ("import faulthandler, signal, time; faulthandler.register(signal.SIGUSR1, all_threads=True);"
            " print('started', flush=True); time.sleep(120)")
    t0 = time.monotonic()
    rc, out, err = _run_phase_process([sys.executable, "-c", hang], None, 2, str(tmp_path), "hang")
    assert rc is None and "started" in out
    assert "most recent call first" in err  # the dumped stack
    assert time.monotonic() - t0 < 30


def test_bench_numa_bind_reports_and_changes_nothing_without_a_gpu():
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    try:
        import bench
    finally:
        sys.path.remove(root)
    import torch

    if torch.cuda.is_available():
        return
    before = os.sched_getaffinity(0)
    r = bench.numa_bind(0)
    assert r["bound"] is False and r["why"] and os.sched_getaffinity(0) == before
