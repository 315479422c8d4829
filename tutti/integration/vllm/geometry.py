"""``tutti.integration.vllm.geometry``: KV geometry of a rank and ``{RANK}``/``{LOCAL_RANK}`` placeholders."""
from tutti_b200.integration.vllm.factory import expand as expand_placeholders  # noqa: F401
from tutti_b200.integration.vllm.factory import geometry_from_layers, parse_bytes  # noqa: F401
from tutti_b200.models.kv_geometry import KVGeometry  # noqa: F401
