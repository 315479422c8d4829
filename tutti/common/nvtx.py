"""``tutti.common.nvtx``: opt-in NVTX ranges (``TUTTI_NVTX=1``), tutti_b200's."""
from tutti_b200.common.observability import nvtx_enabled as enabled  # noqa: F401
from tutti_b200.common.observability import nvtx_range as range  # noqa: F401,A001
