"""Which TP ranks hold identical KV, and which of them reads it (replica IO).

When a model has fewer KV heads than the TP size, each KV head is kept by
``tp // kv_heads`` consecutive ranks: those ranks hold byte-identical main-KV
slices, so one of them (the owner) reads a chunk from SSD and the fused io
kernel stores it into every replica's pool over NVLink. Caches that are the
same on every rank (an MLA latent cache, an index cache) form one group of all
ranks. With decode context parallelism (DCP) the ranks of a group split the
context: main KV then stays rank-local and the replicated caches are shared
only among ranks of the same DCP rank.

The owner of a chunk within a group is ``group[le64(key[:8]) % len(group)]``,
which spreads the reads of a prefix over the group's GPUs.
Parity: reference tutti/integration/vllm/replica_layout.py (validate_replica_io,
replica_groups_for: adjacent-pair groups for duplicated KV heads, all-rank
groups for the index cache, DCP 1 or 2) and replica_direct.py:43-53 (owner
rule); generalised here to any KV-head count and cache kind.
"""
from __future__ import annotations

from typing import Sequence

ENTITY_KINDS = ("main", "latent", "index")


def validate_replica_io(tp: int, kv_heads: int, dp: int = 1, pp: int = 1, dcp: int = 1,
                        gpus_per_node: int = 8) -> None:
    """Raise ValueError when replica IO cannot apply to this parallel layout."""
    if tp < 1 or tp > gpus_per_node:
        raise ValueError(f"replica IO needs single-node TP (1..{gpus_per_node}), got TP{tp}")
    if dp != 1 or pp != 1:
        raise ValueError("replica IO requires DP=1 and PP=1 (replicas are TP ranks of one node)")
    if dcp not in (1, 2) or tp % dcp:
        raise ValueError(f"replica IO supports DCP 1 or 2 dividing TP, got DCP{dcp} at TP{tp}")
    if kv_heads < 1:
        raise ValueError("kv_heads must be positive")
    if kv_heads < tp and tp % kv_heads:
        raise ValueError(f"TP{tp} does not replicate {kv_heads} KV heads evenly")


def replica_group(rank: int, tp: int, kv_heads: int, kind: str = "main", dcp: int = 1) -> tuple[int, ...]:
    """The ranks whose copy of ``kind`` cache is identical to ``rank``'s (including ``rank``)."""
    if kind not in ENTITY_KINDS:
        raise ValueError(f"kind must be one of {ENTITY_KINDS}")
    if not 0 <= rank < tp:
        raise ValueError(f"rank {rank} outside TP{tp}")
    if kind in ("latent", "index"):
        return tuple(r for r in range(tp) if r % dcp == rank % dcp)
    if dcp > 1 or kv_heads >= tp:
        return (rank,)  # every rank has its own heads (or its own context shard)
    rep = tp // kv_heads
    base = rank // rep * rep
    return tuple(range(base, base + rep))


def replica_owner(key: bytes, group: Sequence[int]) -> int:
    """The rank of ``group`` that reads chunk ``key`` for the whole group."""
    group = tuple(group)
    if not group:
        raise ValueError("empty replica group")
    return group[int.from_bytes(bytes(key[:8]), "little") % len(group)]


def read_plan(keys: Sequence[bytes], rank: int, tp: int, kv_heads: int, kind: str = "main",
              dcp: int = 1) -> list[tuple[bytes, int]]:
    """(key, owner) for each chunk this rank needs; owner == rank marks the chunks it reads."""
    g = replica_group(rank, tp, kv_heads, kind, dcp)
    return [(bytes(k), replica_owner(k, g)) for k in keys]
