"""``tutti.engine.completion``: completion handles and the load gate error (tutti_b200's)."""
from tutti_b200.engine.completion import AggregateCompletion, LoadGateError, PostCompletion  # noqa: F401
