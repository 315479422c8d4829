"""``tutti.integration.vllm.connector``: the vLLM v1 KV connector (tutti_b200's)."""
from tutti_b200.integration.vllm.connector import TuttiConnectorV1  # noqa: F401
from tutti_b200.integration.vllm.metadata import TuttiConnectorMetadata  # noqa: F401
