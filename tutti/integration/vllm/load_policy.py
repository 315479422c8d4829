"""``tutti.integration.vllm.load_policy``: sync / async / auto load decisions (tutti_b200's)."""
from tutti_b200.integration.vllm.load_policy import LoadDecision, LoadPolicy, resolve_free_ratio  # noqa: F401
from tutti_b200.integration.vllm.load_policy import LoadPolicy as LoadModePolicy  # noqa: F401
