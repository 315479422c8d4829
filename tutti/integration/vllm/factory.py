"""``tutti.integration.vllm.factory``: connector config and engine construction (tutti_b200's)."""
from tutti_b200.integration.vllm.factory import ConnectorConfig, make_engine  # noqa: F401
