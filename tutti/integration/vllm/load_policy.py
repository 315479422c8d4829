"""``tutti.integration.vllm.load_policy``: sync / async / auto load decisions (tutti_b200's)."""
from tutti_b200.integration.vllm.load_policy import LoadChoice, LoadPolicy, free_ratio_setting  # noqa: F401
from tutti_b200.integration.vllm.load_policy import LoadPolicy as LoadModePolicy  # noqa: F401
