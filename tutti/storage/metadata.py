"""``tutti.storage.metadata``: the scheduler's read-only metadata view of a segment-file namespace."""
from tutti_b200.storage.registry import open_tutti_metadata_view as TuttiMetadataStore  # noqa: F401,N812
