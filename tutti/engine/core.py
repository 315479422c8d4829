"""``tutti.engine.core``: the KV engine (tutti_b200's)."""
from tutti_b200.engine.core import KVEngine  # noqa: F401
