"""``tutti.storage.registry``: store plugins by type name (tutti_b200's; factories take a ``StoreContext``)."""
from tutti_b200.storage.registry import (  # noqa: F401
    StoreContext, create_metadata_store, create_store, register_metadata_store_type, register_store_type,
    store_types)
