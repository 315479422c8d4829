"""Store-type registry: plugin stores selected by a connector config's ``store.type``."""
import sys
import types

import numpy as np
import pytest
import torch

from tutti_b200.index.chunk_index import chunk_keys_for_tokens
from tutti_b200.integration.vllm.factory import ConnectorConfig, make_engine
from tutti_b200.storage import registry
from tutti_b200.storage.memory import MemoryKVStore

SEEN = {}


def _plugin(ctx):
    SEEN["ctx"] = ctx
    store = MemoryKVStore(ctx.geometry.chunk_bytes, capacity_chunks=ctx.capacity_chunks)
    store.open()
    return store


@pytest.fixture(scope="module", autouse=True)
def plugin_type():
    if "test_plugin" not in registry.store_types():
        registry.register_store_type("test_plugin", _plugin)
    yield


def test_plugin_store_type_from_connector_config():
    cfg = ConnectorConfig.from_extra({"chunk_tokens": 32, "store": {
        "type": "test_plugin", "options": {"path": "/kv/{LOCAL_RANK}", "shards": 3}}})
    assert cfg.store_type == "test_plugin" and cfg.store_options == {"path": "/kv/{LOCAL_RANK}", "shards": 3}
    layers = [torch.zeros(2, 8, 16, 2, 64, dtype=torch.bfloat16) for _ in range(2)]
    eng = make_engine(cfg, layers, rank=1, local_rank=1, world=2)
    ctx = SEEN["ctx"]
    assert ctx.options == {"path": "/kv/1", "shards": 3} and (ctx.rank, ctx.world) == (1, 2)
    assert ctx.geometry.num_layers == 2 and eng.staged
    # a chunk round-trips through the plugin store
    for t in layers:
        t.normal_()
    keys = chunk_keys_for_tokens(list(range(32)), 32)
    eng.store_chunks(keys, torch.arange(2)).wait()
    ref = [t[:, :2].clone() for t in layers]
    for t in layers:
        t.zero_()
    eng.load(keys, torch.arange(2)).wait()
    assert all(torch.equal(t[:, :2], r) for t, r in zip(layers, ref))


def test_unknown_and_duplicate_types_are_errors():
    with pytest.raises(ValueError, match="store.type"):
        ConnectorConfig.from_extra({"store": {"type": "no_such_store"}})
    with pytest.raises(ValueError):
        registry.register_store_type("memory", _plugin)
    with pytest.raises(ValueError):
        registry.create_store("no_such_store", None)
    assert {"memory", "tutti", "tutti_nvme", "test_plugin"} <= set(registry.store_types())


def test_metadata_views_resolve_lazily():
    mod = types.ModuleType("tutti_test_meta_plugin")

    class View:
        def __init__(self, options):
            self.options = options

        def recover(self):
            return [b"k" * 16]

    mod.View = View
    sys.modules["tutti_test_meta_plugin"] = mod
    if not registry.has_metadata_store("test_plugin"):
        registry.register_metadata_store_type("test_plugin", "tutti_test_meta_plugin:View")
    v = registry.create_metadata_store("test_plugin", {"root": "/x"})
    assert v.options == {"root": "/x"} and v.recover() == [b"k" * 16]
    with pytest.raises(ValueError):
        registry.register_metadata_store_type("other", "no_colon")
    # the built-in view reports "nothing on media" for a missing namespace
    assert registry.create_metadata_store("tutti", {"root": "/nonexistent/tutti"}) is None


REFERENCE_MODULE_PATHS = {
    "common.errors": ["DirectTransferUnavailable"], "common.nvtx": ["enabled", "range"],
    "common.utils": ["is_int", "positive_int", "parse_capacity", "flatten_block_ids"],
    "engine.completion": ["LoadGateError"], "engine.core": ["KVEngine"],
    "index.chunk_index": [], "integration.vllm.connector": ["TuttiConnectorV1"],
    "integration.vllm.worker": ["WorkerImpl"], "integration.vllm.worker_meta": ["TuttiWorkerMetadata"],
    "integration.vllm.factory": [], "integration.vllm.geometry": ["expand_placeholders"],
    "integration.vllm.green_context": ["enabled", "reserve_io_sms"],
    "integration.vllm.load_policy": ["LoadModePolicy"], "integration.vllm.minimax": [],
    "integration.vllm.replica_layout": ["validate_replica_io"],
    "storage.base": ["KVStore", "Completion"], "storage.memory": ["MemoryKVStore"],
    "storage.registry": ["register_store_type", "register_metadata_store_type", "create_store",
                         "create_metadata_store"],
    "storage.object_store": [], "storage.metadata": ["TuttiMetadataStore"],
    "storage.tutti_nvme.store": ["TuttiKVStore"], "storage.tutti_nvme.object_layout": [],
    "storage.tutti_nvme.layerwise_direct": ["page_geometry"],
    "storage.tutti_nvme.replica_direct": ["owner_index"],
    "storage.tutti_nvme.runtime_factory": ["build_runtime", "prepare_preset", "preset_mounts"],
    "storage.tutti_nvme.preset_derive": ["daemon_config_paths"], "engine.staging": [],
}


def test_reference_module_paths_resolve():
    import importlib

    for mod, names in REFERENCE_MODULE_PATHS.items():
        m = importlib.import_module("tutti." + mod)
        for n in names:
            assert hasattr(m, n), f"tutti.{mod}.{n}"


def test_tutti_store_factory_passes_the_config_through(monkeypatch):
    """The tutti store's constructor arguments, checked with a stand-in class (the real one needs a GPU)."""
    import tutti_b200.storage.tutti_store as ts
    from tutti_b200.models.kv_geometry import KVGeometry

    seen = {}

    class FakeStore:
        def __init__(self, root, geometry, **kw):
            seen.update(root=root, **kw)

        def open(self):
            return self

    monkeypatch.setattr(ts, "TuttiKVStore", FakeStore)
    g = KVGeometry("t", num_layers=2, num_kv_heads=2, head_dim=64, chunk_tokens=32)
    ctx = registry.StoreContext(geometry=g, capacity_chunks=100, namespace=b"ns", device=torch.device("cuda", 3),
                                rank=1, world=2, entity="idx",
                                options={"root": "/kv", "mounts": ["/m0", "/m1"], "segment_file_slots": 64,
                                         "runtime_options": {"leases": 8}, "stored_format": "fp8_block128",
                                         "segment_header_bytes": 8192})
    registry.create_store("tutti_nvme", ctx)
    assert seen["root"] == "/kv/entities/idx" and seen["mounts"] == ["/m0/entities/idx", "/m1/entities/idx"]
    assert seen["device"] == 3 and seen["rank"] == 1 and seen["rank_count"] == 2
    assert seen["segment_file_slots"] == 64 and seen["runtime_options"] == {"leases": 8}
    assert seen["stored_format"] == "fp8_block128" and seen["segment_header_bytes"] == 8192


def test_flatten_block_ids_never_raises():
    import numpy as np

    from tutti.common.utils import flatten_block_ids

    assert flatten_block_ids(None) == ()
    assert flatten_block_ids("abc") == ()
    assert flatten_block_ids(b"\x01\x02") == ()
    assert flatten_block_ids(7) == (7,)
    assert flatten_block_ids([[1, 2], (3,), {4}, 5]) == (1, 2, 3, 4, 5)
    assert flatten_block_ids([[1, [2, 3]], "x", None, np.int64(9)]) == (1, 9)
    assert flatten_block_ids(np.array([[1, 2], [3, 4]])) == ()  # ndarray rows are neither lists nor ints
    assert flatten_block_ids([np.array([1, 2])]) == ()
    assert flatten_block_ids([[np.int32(5), True]]) == (5,)
