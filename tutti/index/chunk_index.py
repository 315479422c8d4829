"""``tutti.index.chunk_index``: chained chunk keys and the residency index (tutti_b200's)."""
from tutti_b200.index.chunk_index import ChunkIndex, chunk_digest, chunk_keys_for_tokens  # noqa: F401
