"""Scheduler side of the vLLM connector: prefix lookup, load decisions, save planning.

The scheduler never touches a file on the request path: residency lives in an
in-memory ``ChunkIndex`` (cold-started from the store's read-only view) and is
updated only when every TP rank reports a chunk committed.

* ``get_num_new_matched_tokens``: chained chunk keys of the prompt (hashed
  incrementally and cached per request), the longest resident prefix, and how
  many of those tokens the engine should load instead of computing (always
  leaving at least one prompt token to compute). The load policy picks a
  synchronous (layerwise, overlapped with the forward) or an asynchronous load.
* ``update_state_after_alloc``: remembers the blocks the loaded chunks land in.
* ``build_meta``: this step's loads, and saves for chunks that become fully
  computed in this step and are not resident (two-phase: plan now, confirm
  from worker metadata).
Parity: reference tutti/integration/vllm/connector.py:421 (get_num_new_matched_tokens),
:678 (build_connector_meta), :808 (update_connector_output), :933-1018 (_lookup_request_prefix).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field

from ...index.chunk_index import ChunkIndex
from .load_policy import LoadPolicy
from .metadata import LoadSpec, SaveSpec, TuttiConnectorMetadata, TuttiWorkerMetadata

LOG = logging.getLogger("tutti_b200.vllm")


@dataclass
class _RequestState:
    keys: list[bytes] = field(default_factory=list)
    parent: bytes | None = None
    hashed_tokens: int = 0
    block_ids: list[int] = field(default_factory=list)
    pending_load: LoadSpec | None = None
    saved_chunks: int = 0  # chunks already planned for saving
    computed_tokens: int = 0


def _tokens(request) -> list[int]:
    for name in ("all_token_ids", "prompt_token_ids"):
        t = getattr(request, name, None)
        if t is not None:
            return list(t)
    raise AttributeError("request has no token ids")


class SchedulerSide:
    def __init__(self, block_size: int, chunk_tokens: int, capacity_chunks: int, tp_size: int = 1,
                 namespace: bytes = b"", policy: LoadPolicy | None = None):
        if chunk_tokens % block_size:
            raise ValueError("chunk_tokens must be a multiple of the engine block size")
        self.block_size = block_size
        self.chunk_tokens = chunk_tokens
        self.blocks_per_chunk = chunk_tokens // block_size
        self.tp_size = tp_size
        self.index = ChunkIndex(capacity_chunks, chunk_tokens, namespace)
        self.policy = policy or LoadPolicy()
        self.requests: dict[str, _RequestState] = {}
        self.generation = 0
        self._planned: dict[bytes, str] = {}  # pending saves: key -> request

    def restore(self, keys) -> None:
        self.index.restore(keys)

    # -- lookup -------------------------------------------------------------
    def _keys(self, req_id: str, tokens: list[int]) -> list[bytes]:
        st = self.requests.setdefault(req_id, _RequestState())
        if st.hashed_tokens + self.chunk_tokens <= len(tokens):
            new, st.parent = self.index.hash_keys(tokens, start=st.hashed_tokens, parent=st.parent)
            st.keys.extend(new)
            st.hashed_tokens += len(new) * self.chunk_tokens
        return st.keys

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> tuple[int, bool]:
        tokens = _tokens(request)
        keys = self._keys(request.request_id, tokens)
        matched = self.index.lookup_prefix_keys(keys)
        # leave at least one prompt token to compute
        limit = ((len(tokens) - 1) // self.chunk_tokens) * self.chunk_tokens
        matched = min(matched, limit)
        ext = max(0, matched - num_computed_tokens)
        # loads start on a chunk boundary
        if num_computed_tokens % self.chunk_tokens:
            ext = 0
        if ext == 0:
            return 0, False
        is_async = self.policy.choose_async(ext)
        return ext, is_async

    def update_state_after_alloc(self, request, block_ids: list[int], num_external_tokens: int,
                                 num_computed_tokens: int = 0, is_async: bool = False) -> None:
        st = self.requests.setdefault(request.request_id, _RequestState())
        st.block_ids = list(block_ids)
        if num_external_tokens <= 0:
            return
        c0 = num_computed_tokens // self.chunk_tokens
        c1 = (num_computed_tokens + num_external_tokens) // self.chunk_tokens
        keys = st.keys[c0:c1]
        blocks = st.block_ids[c0 * self.blocks_per_chunk:c1 * self.blocks_per_chunk]
        if len(blocks) < len(keys) * self.blocks_per_chunk:
            LOG.warning("request %s: %d blocks for %d chunks; skipping load", request.request_id, len(blocks), len(keys))
            return
        self.index.pin(keys)  # protect from eviction while the load is in flight
        st.pending_load = LoadSpec(request.request_id, keys, blocks, num_external_tokens, is_async)

    # -- per step -------------------------------------------------------------
    def build_meta(self, scheduled: list[tuple[str, list[int], int, int]]) -> TuttiConnectorMetadata:
        """``scheduled``: (request id, all block ids, num computed tokens before, num scheduled tokens)."""
        self.generation += 1
        self.index.advance_epoch()
        meta = TuttiConnectorMetadata(generation=self.generation)
        for st_id, st in self.requests.items():
            if st.pending_load is not None:
                meta.loads.append(st.pending_load)
                st.pending_load = None
        for req_id, block_ids, computed, scheduled_tokens in scheduled:
            st = self.requests.get(req_id)
            if st is None:
                continue
            if block_ids:
                st.block_ids = list(block_ids)
            done = computed + scheduled_tokens
            full = min(done // self.chunk_tokens, len(st.keys))
            start = st.saved_chunks
            if full <= start:
                continue
            cand = st.keys[start:full]
            fresh = [k for k in cand if not self.index.is_resident(k) and not self.index.is_pending(k)]
            st.saved_chunks = full
            if not fresh:
                continue
            plan = self.index.plan_store(fresh)
            if plan is None or not plan.new_keys:
                continue
            idx = {k: i for i, k in enumerate(st.keys)}
            blocks = []
            for k in plan.new_keys:
                c = idx[k]
                blocks.extend(st.block_ids[c * self.blocks_per_chunk:(c + 1) * self.blocks_per_chunk])
            for k in plan.new_keys:
                self._planned[k] = req_id
            meta.saves.append(SaveSpec(req_id, list(plan.new_keys), blocks))
        return meta

    def update_from_workers(self, wm: TuttiWorkerMetadata | None) -> list[bytes]:
        """Publish chunks every TP rank committed; returns them."""
        if wm is None:
            return []
        done = [k for k, n in wm.committed.items() if n >= self.tp_size and k in self._planned]
        for k in done:
            self._planned.pop(k, None)
        self.index.confirm_store(done, True)
        return done

    def load_finished(self, request_id: str, keys: list[bytes], ok: bool) -> None:
        try:
            self.index.unpin(keys)
        except KeyError:
            pass
        if not ok:
            self.index.forget(keys)

    def request_finished(self, request_id: str) -> None:
        self.requests.pop(request_id, None)

    def reclaim(self, max_age: int = 64) -> list[bytes]:
        stale = self.index.reclaim_stale_pending(max_age)
        for k in stale:
            self._planned.pop(k, None)
        return stale
