"""``tutti.storage.memory``: the in-process store (tutti_b200's)."""
from tutti_b200.storage.memory import MemoryKVStore  # noqa: F401
