"""``tutti.storage.object_store``: the segment-file object layout (tutti_b200's ``ObjectLayout``)."""
from tutti_b200.storage.object_layout import ObjectLayout, layout_fingerprint  # noqa: F401
