"""``tutti.storage.tutti_nvme.replica_direct``: owner-sharded replica reads fanned out over NVLink (tutti_b200's)."""
from tutti_b200.parallel.fanout import FanoutRestorer, PeerPools, RestoreItem  # noqa: F401
from tutti_b200.parallel.fanout import owner_of as owner_index  # noqa: F401
