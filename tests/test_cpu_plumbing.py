"""CPU plumbing config: POSIX-backed StorageRuntime, Llama-3-8B-shaped paged KV, permuted write and read.

The full configuration is 1,000 blocks (2 GiB of KV); first touches of fresh
memory make that a few minutes on small CI machines, so the suite runs the
same geometry and checks on 96 blocks and ``TUTTI_FULL_PLUMBING=1`` runs 1,000.
"""
import os

from tutti_b200.benchmarks.cpu_plumbing import run


def test_posix_runtime_llama8b_pool_permuted_roundtrip_and_layout(tmp_path):
    blocks = 1000 if os.environ.get("TUTTI_FULL_PLUMBING") == "1" else 96
    r = run(blocks=blocks, seed=0, drives=2, root=str(tmp_path))
    assert r["blocks_equal"], r
    assert r["layout_ok"], r["layout_detail"]
    assert r["bytes"] == blocks * 32 * 65536
