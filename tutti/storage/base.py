"""``tutti.storage.base``: the KV store protocol and completions (tutti_b200's)."""
from tutti_b200.storage.base import Completion, DoneCompletion, KVStore, StoreIOError  # noqa: F401
