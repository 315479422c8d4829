"""NUMA binding of a GPU's host work: CPU-list parsing, the sysfs lookup and the affinity change
(run in a child process so this test process keeps its CPUs)."""
import multiprocessing as mp
import os

from tutti_b200.common import numa


def test_parse_cpulist():
    assert numa.parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert numa.parse_cpulist("") == [] and numa.parse_cpulist("5") == [5]


def test_local_cpus_reads_the_pci_function(tmp_path):
    d = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    d.mkdir(parents=True)
    (d / "local_cpulist").write_text("0-1,4\n")
    assert numa.local_cpus("0000:1B:00.0", str(tmp_path)) == [0, 1, 4]
    assert numa.local_cpus("0000:99:00.0", str(tmp_path)) == []


def _child(q, cpus):
    applied = numa.bind_cpus(cpus)
    q.put((applied, sorted(os.sched_getaffinity(0))))


def test_bind_cpus_intersects_with_the_allowed_set():
    allowed = sorted(os.sched_getaffinity(0))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(q, [allowed[0], 10_000]))
    p.start()
    applied, now = q.get(timeout=60)
    p.join(30)
    assert applied == [allowed[0]] and now == [allowed[0]]
    p = ctx.Process(target=_child, args=(q, [10_000]))  # nothing allowed: unchanged
    p.start()
    applied, now = q.get(timeout=60)
    p.join(30)
    assert applied == [] and now == allowed


def test_bind_to_gpu_without_cuda_changes_nothing():
    import torch

    if torch.cuda.is_available():
        return
    before = os.sched_getaffinity(0)
    r = numa.bind_to_gpu(0)
    assert r["bound"] is False and os.sched_getaffinity(0) == before
