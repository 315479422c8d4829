"""``tutti.storage.tutti_nvme.layerwise_direct``: per-layer page geometry on media (tutti_b200's)."""
from tutti_b200.storage.tutti_store import stored_geometry as page_geometry  # noqa: F401
