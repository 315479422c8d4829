"""``tutti.integration.vllm.minimax``: several KV entities per layer (main KV + index cache), tutti_b200's."""
from tutti_b200.engine.entities import EntityEngines  # noqa: F401
