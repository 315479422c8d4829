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
* ``update_from_workers``: publishes chunks every TP rank committed, settles
  loads (a synchronous load with the step it ran in, an asynchronous one when
  vLLM reports it received): the chunks are unpinned, and those from a failed
  chunk on are forgotten; feeds the workers' read and step measurements to the
  load policy.
The block usage the policy needs is estimated from the live requests (vLLM's
pool is not visible here): each running request holds ceil(computed tokens /
block size) blocks, an asynchronous load holds its allocated blocks.
Parity: reference tutti/integration/vllm/connector.py:421 (get_num_new_matched_tokens),
:678 (build_connector_meta), :808 (update_connector_output), :933-1018
(_lookup_request_prefix), :1032-1062 (_block_usage).
"""
from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field

from ...common.observability import health_interval_s
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
                 namespace: bytes = b"", policy: LoadPolicy | None = None, total_blocks: int | None = None,
                 log_interval_s: float | None = None, min_retrieve_tokens: int = 0, max_tokens_per_load: int = 0):
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
        self._saving_requests: set[str] = set()  # requests that had a save
        self._finished_saving: set[str] = set()  # ... and finished since the last step
        self.total_blocks = total_blocks  # vLLM's KV pool size, when known
        self.min_retrieve_tokens = min_retrieve_tokens  # shorter hits are computed instead
        self.max_tokens_per_load = max_tokens_per_load  # 0: no cap
        self._live: dict[str, object] = {}  # request objects, for the block-usage estimate
        self._async_blocks: dict[str, int] = {}  # asynchronous loads not yet received -> blocks held
        self._sync_loads: dict[int, list[tuple[str, list[bytes]]]] = {}  # generation -> loads dispatched
        self._async_loads: dict[str, list[bytes]] = {}  # request -> keys of its dispatched async load
        self._log_interval = (health_interval_s() if log_interval_s is None
                              else log_interval_s)
        self._last_log = time.monotonic()
        self.profile = {"lookups": 0, "hit_tokens": 0, "hash_ms": 0.0, "loads_ok": 0, "loads_failed": 0}

    def restore(self, keys) -> None:
        self.index.restore(keys)

    # -- lookup -------------------------------------------------------------
    def _keys(self, req_id: str, tokens: list[int]) -> list[bytes]:
        st = self.requests.setdefault(req_id, _RequestState())
        if st.hashed_tokens + self.chunk_tokens <= len(tokens):
            t0 = time.perf_counter()
            new, st.parent = self.index.hash_keys(tokens, start=st.hashed_tokens, parent=st.parent)
            self.profile["hash_ms"] += (time.perf_counter() - t0) * 1e3
            st.keys.extend(new)
            st.hashed_tokens += len(new) * self.chunk_tokens
        return st.keys

    def _block_usage(self, req_id: str) -> tuple[int, int, int | None]:
        """(other running requests, blocks held by asynchronous loads, estimated free blocks or None).

        Preempted requests and shared prefix blocks are counted as used, which
        errs towards fewer free blocks, i.e. towards synchronous loads.
        """
        held = sum(self._async_blocks.values())
        others = used = 0
        for rid, req in self._live.items():
            if rid == req_id or rid in self._async_blocks:
                continue
            status = getattr(req, "status", None)
            if status is not None and getattr(status, "name", str(status)) != "RUNNING":
                continue
            others += 1
            used += -(-int(getattr(req, "num_computed_tokens", 0) or 0) // self.block_size)
        free = None if not self.total_blocks else int(self.total_blocks) - used - held
        return others, held, free

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> tuple[int, bool]:
        tokens = _tokens(request)
        keys = self._keys(request.request_id, tokens)
        matched = self.index.lookup_prefix_keys(keys)
        self.profile["lookups"] += 1
        # leave at least one prompt token to compute
        limit = ((len(tokens) - 1) // self.chunk_tokens) * self.chunk_tokens
        matched = min(matched, limit)
        ext = max(0, matched - num_computed_tokens)
        # loads start on a chunk boundary
        if num_computed_tokens % self.chunk_tokens:
            ext = 0
        if self.min_retrieve_tokens and ext < self.min_retrieve_tokens:
            ext = 0
        if self.max_tokens_per_load:
            ext = min(ext, self.max_tokens_per_load // self.chunk_tokens * self.chunk_tokens)
        if ext == 0:
            return 0, False
        self.profile["hit_tokens"] += ext
        others, held, free = self._block_usage(request.request_id)
        decision = self.policy.decide(chunks=ext // self.chunk_tokens,
                                      compute_tokens=len(tokens) - num_computed_tokens - ext, others=others,
                                      held_blocks=held, need_blocks=-(-(num_computed_tokens + ext) // self.block_size),
                                      free_blocks=free)
        return ext, decision.asynchronous

    def update_state_after_alloc(self, request, block_ids: list[int], num_external_tokens: int,
                                 num_computed_tokens: int = 0, is_async: bool = False) -> None:
        st = self.requests.setdefault(request.request_id, _RequestState())
        st.block_ids = list(block_ids)
        self._live[request.request_id] = request
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
        if is_async:
            self._async_blocks[request.request_id] = len(blocks)

    # -- per step -------------------------------------------------------------
    def build_meta(self, scheduled: list[tuple[str, list[int], int, int]],
                   step_tokens: int | None = None) -> TuttiConnectorMetadata:
        """``scheduled``: (request id, all block ids, num computed tokens before, num scheduled tokens)."""
        self.generation += 1
        self.index.advance_epoch()
        self.reclaim()
        meta = TuttiConnectorMetadata(generation=self.generation,
                                      step_tokens=sum(s[3] for s in scheduled) if step_tokens is None else step_tokens,
                                      finished_saving=sorted(self._finished_saving))
        self._finished_saving.clear()
        for st_id, st in self.requests.items():
            if st.pending_load is not None:
                ld = st.pending_load
                meta.loads.append(ld)
                st.pending_load = None
                if ld.is_async:
                    self._async_loads[ld.request_id] = list(ld.keys)
                else:
                    self._sync_loads.setdefault(self.generation, []).append((ld.request_id, list(ld.keys)))
        self.maybe_log()
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
            self._saving_requests.add(req_id)
        return meta

    def update_from_workers(self, wm: TuttiWorkerMetadata | None, finished_recving=()) -> list[bytes]:
        """Publish chunks every TP rank committed (returned); settle finished loads; feed the policy."""
        failed = dict(wm.failed_loads) if wm is not None else {}
        # asynchronous loads vLLM reports received (on every rank)
        for rid in finished_recving or ():
            keys = self._async_loads.pop(rid, None)
            self._async_blocks.pop(rid, None)
            if keys is not None:
                self.load_finished(rid, keys, rid not in failed, failed.get(rid, 0))
        if wm is None:
            return []
        # synchronous loads settle with the step they ran in (and any older step left unreported)
        for gen in [g for g in self._sync_loads if g <= wm.generation]:
            for rid, keys in self._sync_loads.pop(gen):
                self.load_finished(rid, keys, rid not in failed, failed.get(rid, 0))
        # TP ranks advance together: each step follows its slowest rank
        reads = [(int(c), float(ms)) for c, ms in wm.read_samples if c > 0 and ms > 0]
        if reads:
            self.policy.record_restore(*max(reads, key=lambda x: x[1] / x[0]))
        steps = [(int(t), float(ms)) for t, ms in wm.step_samples if t > 0 and ms > 0]
        if steps:
            self.policy.record_step(*max(steps, key=lambda x: x[1]))
        done = [k for k, n in wm.committed.items() if n >= self.tp_size and k in self._planned]
        for k in done:
            self._planned.pop(k, None)
        self.index.confirm_store(done, True)
        return done

    def load_finished(self, request_id: str, keys: list[bytes], ok: bool, first_failed_token: int = 0) -> None:
        """Unpin a finished load's chunks; after a failure forget those from the failed chunk on."""
        try:
            self.index.unpin(keys)
        except KeyError:
            pass
        self.profile["loads_ok" if ok else "loads_failed"] += 1
        if not ok:
            self.index.forget(keys[max(0, first_failed_token) // self.chunk_tokens:])

    def request_finished(self, request_id: str) -> bool:
        """Forget the request. Its blocks are freed at once; if it had saves, the next step's
        metadata names it, and the workers order that step's forward after those saves on
        the device (a freed block may be written again only once the saves read it).
        Returns False: no delayed free."""
        self.requests.pop(request_id, None)
        self._live.pop(request_id, None)
        if request_id in self._saving_requests:
            self._saving_requests.discard(request_id)
            self._finished_saving.add(request_id)
        return False

    def maybe_log(self, force: bool = False) -> bool:
        """``[tutti] index-profile`` and ``[tutti] load-policy`` lines, at most once per interval."""
        now = time.monotonic()
        if not force and now - self._last_log < self._log_interval:
            return False
        self._last_log = now
        p, st = self.profile, self.index.stats() if hasattr(self.index, "stats") else {}
        LOG.info("[tutti] index-profile lookups=%d hit_tokens=%d hash_ms=%.1f loads_ok=%d loads_failed=%d %s",
                 p["lookups"], p["hit_tokens"], p["hash_ms"], p["loads_ok"], p["loads_failed"],
                 " ".join(f"{k}={v}" for k, v in st.items()))
        snap = self.policy.snapshot()
        LOG.info("[tutti] load-policy " + " ".join(f"{k}={v}" for k, v in snap.items()))
        return True

    def reclaim(self, max_age: int = 64) -> list[bytes]:
        stale = self.index.reclaim_stale_pending(max_age)
        for k in stale:
            self._planned.pop(k, None)
        return stale
