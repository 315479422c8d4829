"""``tutti.integration.vllm.worker_meta``: per-step worker metadata (tutti_b200's)."""
from tutti_b200.integration.vllm.metadata import TuttiWorkerMetadata  # noqa: F401
