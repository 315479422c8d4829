"""``tutti.integration.vllm.replica_layout``: replica groups, owners and validation (tutti_b200's)."""
from tutti_b200.parallel.replica_layout import read_plan, replica_group, replica_owner, validate_replica_io  # noqa: F401
