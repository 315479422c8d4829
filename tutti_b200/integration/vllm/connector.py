"""TuttiConnectorV1: vLLM v1 KV connector backed by the tutti_b200 store.

Use with vLLM:
    --kv-transfer-config '{"kv_connector": "TuttiConnectorV1",
        "kv_connector_module_path": "tutti_b200.integration.vllm.connector",
        "kv_role": "kv_both",
        "kv_connector_extra_config": {"chunk_tokens": 256, "store": {"root": "/mnt/kv/{LOCAL_RANK}"}}}'

Scheduler role: prefix lookup over chained chunk keys, load decisions,
save planning, publication of chunks committed by every TP rank.
Worker role: layerwise restores overlapped with the forward
(``wait_for_layer_load``), saves after the forward (``wait_for_save``), TP
failure consensus and load-error reporting.
Parity: reference tutti/integration/vllm/connector.py:178-1067.
"""
from __future__ import annotations

import logging
import os
from typing import Any

from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1, KVConnectorRole

from .factory import ConnectorConfig, make_engine
from .load_policy import LoadPolicy
from .metadata import TuttiConnectorMetadata, TuttiWorkerMetadata
from .scheduler import SchedulerSide
from .worker import WorkerSide

LOG = logging.getLogger("tutti_b200.vllm")


def _tp_info():
    try:
        from vllm.distributed.parallel_state import get_tp_group

        g = get_tp_group()
        return g.rank_in_group, g.world_size, g.cpu_group
    except Exception:  # noqa: BLE001 - no distributed state (tests, single process)
        return 0, 1, None


def _uses_mla(vllm_config) -> bool:
    return bool(getattr(getattr(vllm_config, "model_config", None), "use_mla", False))


def _total_kv_heads(vllm_config) -> int | None:
    """The model's KV-head count (all TP ranks), or None when vLLM does not say."""
    mc = getattr(vllm_config, "model_config", None)
    try:
        return int(mc.get_total_num_kv_heads())
    except Exception:  # noqa: BLE001 - replica groups then default to one rank each
        return None


class TuttiConnectorV1(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        ktc = vllm_config.kv_transfer_config
        extra = getattr(ktc, "kv_connector_extra_config", None) or {}
        self.cfg = ConnectorConfig.from_extra(extra)
        vllm_policy = getattr(ktc, "kv_load_failure_policy", None)
        if vllm_policy and "kv_load_failure_policy" in extra and extra["kv_load_failure_policy"] != vllm_policy:
            LOG.warning("[tutti] kv_load_failure_policy %r in the connector config is ignored: vLLM applies "
                        "its own kv_transfer_config.kv_load_failure_policy (%r)", extra["kv_load_failure_policy"],
                        vllm_policy)
        cache = vllm_config.cache_config
        self.block_size = int(cache.block_size)
        par = vllm_config.parallel_config
        self.tp_size = int(getattr(par, "tensor_parallel_size", 1))
        self._sched: SchedulerSide | None = None
        self._worker: WorkerSide | None = None
        if role == KVConnectorRole.SCHEDULER:
            capacity = self.cfg.capacity_chunks or 1 << 20
            total_blocks = getattr(kv_cache_config, "num_blocks", None) if kv_cache_config is not None else None
            self._sched = SchedulerSide(self.block_size, self.cfg.chunk_tokens, capacity, self.tp_size,
                                        namespace=self.cfg.namespace.encode(),
                                        policy=LoadPolicy(self.cfg.load_mode, free_ratio=self.cfg.async_load_free_ratio),
                                        total_blocks=total_blocks, min_retrieve_tokens=self.cfg.min_retrieve_tokens,
                                        max_tokens_per_load=self.cfg.max_tokens_per_load)
            self._async_pending: dict[str, bool] = {}
            self._cold_start()
        else:
            rank, world, cpu_group = _tp_info()
            from ...parallel.tp_consensus import TpFailureConsensus

            local_rank = int(os.environ.get("LOCAL_RANK", rank))
            self._worker = WorkerSide(lambda tensors, entity="": make_engine(self.cfg, tensors, rank, local_rank,
                                                                             world, entity),
                                      block_size=self.block_size, chunk_tokens=self.cfg.chunk_tokens,
                                      tp_rank=rank, tp_size=world, consensus=TpFailureConsensus(cpu_group, self.cfg.failure_timeout_s),
                                      # vLLM's scheduler applies kv_load_failure_policy (recompute or fail the
                                      # requests) to the blocks the worker reports; the worker only reports
                                      failure_policy="recompute", lookahead=self.cfg.lookahead_k,
                                      max_inflight_saves=self.cfg.max_inflight_saves,
                                      replica_io=self.cfg.replica_io, group=cpu_group,
                                      replica_kind="latent" if _uses_mla(vllm_config) else "main",
                                      kv_heads=_total_kv_heads(vllm_config),
                                      replica_io_saves=self.cfg.replica_io_saves)

    def _cold_start(self) -> None:
        """Publish the chunks a previous run left in the store (a read-only view; no model geometry needed)."""
        from ...storage.registry import create_metadata_store, has_metadata_store
        from .factory import expand

        if not has_metadata_store(self.cfg.store_type):
            return
        if self.cfg.store_type == "tutti":
            options = {"root": expand(self.cfg.root, 0, 0), "mounts": [expand(m, 0, 0) for m in self.cfg.mounts],
                       "rank": 0}
        else:
            options = {k: expand(v, 0, 0) if isinstance(v, str) else v for k, v in self.cfg.store_options.items()}
        try:
            view = create_metadata_store(self.cfg.store_type, options)
            if view is None:
                return
            keys = view.recover()
            if self.tp_size > 1:  # resident only where every TP rank holds its slice
                keys = [k for k in keys if view.contains_prefix([k], True) == 1]
            view.close()
        except Exception as e:  # noqa: BLE001 - a cold store only costs recomputation
            LOG.warning("[tutti] cold start skipped: %s", e)
            return
        self._sched.restore(keys)
        LOG.info("[tutti] cold start: %d resident chunk(s)", len(keys))

    # ---------------- scheduler role ----------------
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        ext, is_async = self._sched.get_num_new_matched_tokens(request, num_computed_tokens)
        self._async_pending[request.request_id] = is_async
        return ext, is_async

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        block_ids = list(blocks.get_block_ids()[0]) if blocks is not None else []
        self._sched.update_state_after_alloc(request, block_ids, num_external_tokens,
                                             getattr(request, "num_computed_tokens", 0),
                                             self._async_pending.pop(request.request_id, False))

    def build_connector_meta(self, scheduler_output) -> TuttiConnectorMetadata:
        scheduled = []
        for nr in getattr(scheduler_output, "scheduled_new_reqs", []):
            n = scheduler_output.num_scheduled_tokens.get(nr.req_id, 0)
            scheduled.append((nr.req_id, list(nr.block_ids[0]) if nr.block_ids else [], nr.num_computed_tokens, n))
        cached = getattr(scheduler_output, "scheduled_cached_reqs", None)
        if cached is not None:
            for i, rid in enumerate(cached.req_ids):
                n = scheduler_output.num_scheduled_tokens.get(rid, 0)
                new_blocks = cached.new_block_ids[i]
                st = self._sched.requests.get(rid)
                blocks = list(st.block_ids) if st else []
                if new_blocks:
                    blocks += list(new_blocks[0])
                scheduled.append((rid, blocks, cached.num_computed_tokens[i], n))
        return self._sched.build_meta(scheduled, getattr(scheduler_output, "total_num_scheduled_tokens", None))

    def update_connector_output(self, connector_output) -> None:
        wm = getattr(connector_output, "kv_connector_worker_meta", None)
        received = getattr(connector_output, "finished_recving", None) or ()
        self._sched.update_from_workers(wm if isinstance(wm, TuttiWorkerMetadata) else None, received)

    def request_finished(self, request, block_ids: list[int]) -> tuple[bool, dict[str, Any] | None]:
        # blocks are freed now; the next step's forward is ordered after the
        # request's saves on the device (see TuttiConnectorMetadata.finished_saving)
        return self._sched.request_finished(request.request_id), None

    # ---------------- worker role ----------------
    def register_kv_caches(self, kv_caches) -> None:
        self._worker.register_kv_caches(kv_caches)

    def start_load_kv(self, forward_context, **kwargs) -> None:
        meta = self._get_connector_metadata()
        assert isinstance(meta, TuttiConnectorMetadata)
        self._worker.start_load_kv(meta)

    def wait_for_layer_load(self, layer_name: str) -> None:
        self._worker.wait_for_layer_load(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer, attn_metadata, **kwargs) -> None:
        return None  # the whole step's chunks are saved in wait_for_save, behind one compute event

    def wait_for_save(self) -> None:
        meta = self._get_connector_metadata()
        self._last_worker_meta = self._worker.wait_for_save(meta)

    def build_connector_worker_meta(self):
        # once per step: a step without wait_for_save must not resend the last one's commits
        meta, self._last_worker_meta = getattr(self, "_last_worker_meta", None), None
        return meta

    def get_finished(self, finished_req_ids: set[str]):
        return self._worker.get_finished(finished_req_ids)

    def get_block_ids_with_load_errors(self) -> set[int]:
        return self._worker.get_block_ids_with_load_errors()

    def shutdown(self):
        if self._worker is not None:
            self._worker.shutdown()
