"""Tensor-parallel load-failure consensus.

Each TP rank restores its own KV-head slice. If any rank fails to load part of
a request's prefix, every rank must treat the same chunk range as failed (and
recompute it), or the ranks would attend over different context. After a
step with external loads, ranks exchange one fixed-size int64 row over a CPU
(gloo) process group:

    row = [generation, first_0, end_0, first_1, end_1, ...]   (-1, -1: no failure)

and merge them: a request's failed range is the union (min first, max end) of
the ranks' ranges; a row with another generation makes the step inconsistent
(treated as failed). A second fixed collective (``drain_barrier``) runs only
after a global failure, so every rank drains its in-flight IO before the
failed blocks are reused. Both collectives carry a timeout, so a rank that
died makes the others fail loudly instead of hanging.
Parity: reference tutti/integration/vllm/worker.py:128-238
(_TpLoadFailureCoordinator.coordinate / merge_rows / drain_barrier).
"""
from __future__ import annotations

import datetime
import time
from dataclasses import dataclass
from typing import Iterable, Sequence

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ChunkFailure:
    request: int      # ordinal of the request in this step's load list
    first_chunk: int  # first failed chunk ordinal within the request's loaded chunks
    count: int


@dataclass(frozen=True)
class Consensus:
    failed: bool
    generation: int
    consistent: bool
    failures: tuple[ChunkFailure, ...]
    latency_ms: float = 0.0

    def failed_chunks(self, request: int) -> range:
        for f in self.failures:
            if f.request == request:
                return range(f.first_chunk, f.first_chunk + f.count)
        return range(0)


def encode_row(generation: int, n_requests: int, failures: Iterable[ChunkFailure]) -> list[int]:
    row = [int(generation)] + [-1] * (2 * n_requests)
    for f in failures:
        if not 0 <= f.request < n_requests or f.count <= 0:
            raise ValueError(f"bad failure record {f}")
        first, end = f.first_chunk, f.first_chunk + f.count
        cur_first, cur_end = row[1 + 2 * f.request], row[2 + 2 * f.request]
        if cur_first >= 0:
            first, end = min(first, cur_first), max(end, cur_end)
        row[1 + 2 * f.request], row[2 + 2 * f.request] = first, end
    return row


def merge_rows(generation: int, n_requests: int, rows: Sequence[Sequence[int]], latency_ms: float = 0.0) -> Consensus:
    consistent = all(int(r[0]) == generation for r in rows) and all(len(r) == 1 + 2 * n_requests for r in rows)
    merged: dict[int, tuple[int, int]] = {}
    for r in rows:
        if len(r) != 1 + 2 * n_requests:
            continue
        for q in range(n_requests):
            first, end = int(r[1 + 2 * q]), int(r[2 + 2 * q])
            if first < 0 or end <= first:
                continue
            prev = merged.get(q)
            merged[q] = (first, end) if prev is None else (min(prev[0], first), max(prev[1], end))
    failures = tuple(ChunkFailure(q, a, b - a) for q, (a, b) in sorted(merged.items()))
    return Consensus(bool(failures) or not consistent, generation, consistent, failures, latency_ms)


class TpFailureConsensus:
    """Runs the two collectives on a CPU process group (gloo); world size 1 needs no collective."""

    def __init__(self, group=None, timeout_s: float = 30.0):
        if timeout_s <= 0:
            raise ValueError("timeout must be positive")
        self.group = group
        self.timeout = datetime.timedelta(seconds=timeout_s)

    def _world(self) -> int:
        if not dist.is_available() or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.group)

    def _gather(self, local: torch.Tensor) -> list[list[int]]:
        world = self._world()
        out = torch.empty(world * local.numel(), dtype=torch.int64)
        work = dist.all_gather_into_tensor(out, local, group=self.group, async_op=True)
        if work.wait(timeout=self.timeout) is False:
            raise TimeoutError(f"TP consensus collective timed out after {self.timeout.total_seconds()} s")
        return out.reshape(world, local.numel()).tolist()

    def coordinate(self, generation: int, n_requests: int, failures: Iterable[ChunkFailure]) -> Consensus:
        failures = list(failures)
        row = encode_row(generation, n_requests, failures)
        if self._world() <= 1:
            return merge_rows(generation, n_requests, [row])
        t0 = time.monotonic_ns()
        rows = self._gather(torch.tensor(row, dtype=torch.int64))
        return merge_rows(generation, n_requests, rows, (time.monotonic_ns() - t0) / 1e6)

    def drain_barrier(self, generation: int, local_ok: bool) -> bool:
        if self._world() <= 1:
            return bool(local_ok)
        rows = self._gather(torch.tensor([generation, int(bool(local_ok))], dtype=torch.int64))
        return all(int(r[0]) == generation and int(r[1]) == 1 for r in rows)
