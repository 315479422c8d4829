"""``tutti.storage.tutti_nvme.store``: the NVMe-backed KV store (tutti_b200's)."""
from tutti_b200.storage.tutti_store import NativeCompletion, TuttiKVStore  # noqa: F401
