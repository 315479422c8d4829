"""Exceptions shared across layers.

``DirectTransferUnavailable``: a direct (paged) transfer was asked of a store
that only moves chunks through staging buffers.
Parity: reference tutti/common/errors.py (DirectTransferUnavailable).
"""
from __future__ import annotations

from ..engine.completion import LoadGateError  # noqa: F401
from ..storage.base import StoreIOError  # noqa: F401


class DirectTransferUnavailable(NotImplementedError):
    pass
