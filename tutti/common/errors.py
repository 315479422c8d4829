"""``tutti.common.errors`` (tutti_b200's)."""
from tutti_b200.common.errors import DirectTransferUnavailable, LoadGateError, StoreIOError  # noqa: F401
