"""Loader for the in-tree native extensions.

``core()`` returns ``tutti_b200._core`` (runtime, object store, NVMe data
paths); ``ops()`` returns ``tutti_b200._ops`` (torch-facing sm_100a kernels).
Both are built in place by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``). On a machine with a CUDA device a missing
extension is an error, never a silent fallback.
"""
from __future__ import annotations

import importlib

_CACHE: dict[str, object] = {}


class NativeExtensionMissing(ImportError):
    pass


def _load(name: str):
    if name in _CACHE:
        return _CACHE[name]
    import torch  # noqa: F401  (loads the CUDA runtime the extensions link against)

    try:
        mod = importlib.import_module(f"tutti_b200.{name}")
    except ImportError as e:  # pragma: no cover - exercised only without a build
        raise NativeExtensionMissing(
            f"tutti_b200.{name} is not built; run `python setup.py build_ext --inplace`"
        ) from e
    _CACHE[name] = mod
    return mod


def core():
    return _load("_core")


def ops():
    return _load("_ops")


def have_ops() -> bool:
    try:
        ops()
        return True
    except NativeExtensionMissing:
        return False
