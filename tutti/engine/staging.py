"""``tutti.engine.staging``: reused staging memory of the staged path (tutti_b200's ``StagingBuffer``)."""
from tutti_b200.engine.staging import StagingBuffer  # noqa: F401
