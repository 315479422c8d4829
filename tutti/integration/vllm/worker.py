"""``tutti.integration.vllm.worker``: the connector's worker side (``WorkerImpl`` is tutti_b200's ``WorkerSide``)."""
from tutti_b200.integration.vllm.worker import WorkerSide, normalize_kv_layer  # noqa: F401
from tutti_b200.integration.vllm.worker import WorkerSide as WorkerImpl  # noqa: F401
