"""``tutti.storage.tutti_nvme.object_layout``: segment-file layout (tutti_b200's)."""
from tutti_b200.storage.object_layout import ObjectLayout, layout_fingerprint  # noqa: F401
