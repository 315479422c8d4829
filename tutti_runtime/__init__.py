"""``tutti_runtime``: Tutti's Python binding surface over tutti_b200's native runtime.

    make_stub_runtime(accel_id=-1) -> Runtime
    make_local_nvme_runtime(preset) / make_nvme_device_group_runtime(preset) /
    make_raid0_nvme_runtime(preset) -> Runtime
    Runtime: caps / open_batch / close_target / close_batch / register_memory /
             unregister_memory / submit / enqueue_wait / release_io / query_io /
             open_io_count / wait / wait_result / wait_detail / shutdown /
             testing_force_complete (stub runtimes: their IOs wait for it)
    SubmitResult, WaitResult
    ObjectStore: open(scheme, config) / contains_prefix_all_ranks / lookup / usage / ...

Presets take Tutti's form (``tutti_b200.storage.preset``): the drives' mounts are
given in the preset or derived from its daemon configuration, and each mount is
served by one NVMe controller of this build's GPU data path. A request is a
6-tuple ``(target, target_offset, memory, memory_offset, length, "read"|"write")``;
one submit may mix reads and writes. Terminal results stay readable after
``release_io`` (``wait_result`` / ``query_io``).
Parity: reference csrc/python/src/tutti_runtime/__init__.py and
csrc/python/src/_core.cpp:83-110 (SubmitResult, WaitResult), :254-400 (submit,
query_io, wait, wait_result), :1228-1313 (Runtime methods, factories).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field

import numpy as np

from tutti_b200._native import core as _core
from tutti_b200.storage.preset import prepare_preset, preset_mounts

__all__ = ["Runtime", "ObjectStore", "SubmitResult", "WaitResult", "make_stub_runtime", "make_local_nvme_runtime",
           "make_nvme_device_group_runtime", "make_raid0_nvme_runtime"]


@dataclass
class SubmitResult:
    status_ok: bool
    status_msg: str
    io_handle: int | None  # None: every request was rejected
    initial_states: list[bool] = field(default_factory=list)  # True: accepted
    rejected: list[int] = field(default_factory=list)  # request indices to resubmit


@dataclass
class WaitResult:
    observation: str  # OK | TIMEOUT
    state: str  # COMPLETED | FAILED | IN_FLIGHT
    confirmed_bytes: int = 0
    timeout_seen: bool = False
    failed_request_indices: list[int] = field(default_factory=list)
    failure_scope: str = "NONE"
    failure_kind: str | None = None
    first_failed_entry: int | None = None
    raw_cq_status: int | None = None
    message: str = ""


def _runtime_from_preset(preset: dict, kind: str) -> "Runtime":
    p = dict(preset)
    p.setdefault("type", kind)
    prepared = prepare_preset(p)
    accel = prepared.get("gpu_id", 0)
    accel = int(accel) if isinstance(accel, int) or str(accel).isdigit() else 0
    options = {k: prepared[k] for k in ("leases", "max_ctas_per_op", "slots_per_lease", "timeout_ms") if k in prepared}
    return Runtime(_core().make_emulated_nvme_runtime(accel, preset_mounts(prepared), options))


def make_stub_runtime(accel_id: int = -1) -> "Runtime":
    """A runtime with no storage components: memory verbs work, open/submit report errors."""
    return Runtime(_core().make_stub_runtime(accel_id))


def make_local_nvme_runtime(preset: dict) -> "Runtime":
    return _runtime_from_preset(preset, "local")


def make_nvme_device_group_runtime(preset: dict) -> "Runtime":
    return _runtime_from_preset(preset, "nvme-device-group")


def make_raid0_nvme_runtime(preset: dict) -> "Runtime":
    return _runtime_from_preset(preset, "raid0")


_KINDS = {"device": "device", "host": "host", "pinned": "pinned", "pinned_host": "pinned"}


class Runtime:
    """Tutti's ``Runtime`` methods over a tutti_b200 runtime (``tutti_b200._core.Runtime``)."""

    RETAINED = 4096  # terminal results kept for reading after release_io (oldest dropped first)

    def __init__(self, native):
        self.native = native
        self._open: set[int] = set()  # submitted, not yet released
        self._retained: dict[int, WaitResult] = {}  # terminal results, kept after release_io

    # -- capabilities, targets, memory ---------------------------------------------
    def caps(self):
        return self.native.caps()

    def open_batch(self, uris):
        return self.native.open_batch(list(uris))

    def close_target(self, target_handle: int) -> None:
        self.native.close(int(target_handle))

    def close_batch(self, target_handles) -> None:
        for h in target_handles:
            self.native.close(int(h))

    def register_memory(self, addr: int, size: int, kind: str, accel_id: int = -1, io_granularity: int = 0) -> int:
        k = _KINDS.get(str(kind).lower())
        if k is None:
            raise ValueError(f"memory kind must be one of {sorted(_KINDS)}, got {kind!r}")
        return self.native.register_memory(int(addr), int(size), k, int(accel_id), int(io_granularity))

    def unregister_memory(self, memory_ticket: int) -> None:
        self.native.unregister_memory(int(memory_ticket))

    # -- IO -------------------------------------------------------------------------
    def submit(self, requests, accel_id: int, stream, execution: str = "device") -> SubmitResult:
        """``requests``: 6-tuples (target, target_offset, memory, memory_offset, length, "read"|"write")."""
        if execution not in ("device", "host"):
            raise ValueError(f"execution must be 'device' or 'host', got {execution!r}")
        if execution == "device" and stream is None:
            raise ValueError("execution='device' requires a stream (a cudaStream_t pointer)")
        reqs = list(requests)
        if any(len(r) != 6 for r in reqs):
            raise ValueError("each request must be a 6-tuple")
        a = lambda i: np.asarray([r[i] for r in reqs], dtype=np.uint64)  # noqa: E731
        dirs = [r[5] for r in reqs]
        if any(d not in ("read", "write") for d in dirs):
            raise ValueError("request direction must be 'read' or 'write'")
        kinds = set(dirs)
        direction = kinds.pop() if len(kinds) == 1 else "mixed"
        out = self.native.submit_arrays(direction, a(2), a(3), a(0), a(1), a(4), int(stream or 0), execution == "host",
                                        np.asarray([d == "write" for d in dirs], dtype=np.uint8))
        rejected = [int(i) for i in out["rejected"]]
        io = out["io"]
        if io is not None:
            self._open.add(int(io))
        bad = set(rejected)
        return SubmitResult(bool(out["ok"]), out["status"], None if io is None else int(io),
                            [i not in bad for i in range(len(reqs))], rejected)

    def enqueue_wait(self, io_handles, stream) -> None:
        self.native.enqueue_wait([int(h) for h in io_handles], int(stream))

    def wait_result(self, io_handle: int, timeout_ms: int = 0) -> WaitResult:
        h = int(io_handle)
        if h in self._retained:
            return self._retained[h]
        r = self.native.wait(h, int(timeout_ms))
        if r is None:
            return WaitResult("TIMEOUT", "IN_FLIGHT")
        failed = list(r["failed_request_indices"])
        res = WaitResult("OK", str(r["state"]).upper(), int(r["confirmed_bytes"]), bool(r["timeout_seen"]), failed,
                         "REQUEST_INDICES" if failed else ("NONE" if r["ok"] else "WHOLE_OPERATION"),
                         None if r["ok"] else str(r["failure_kind"]).upper(), failed[0] if failed else None,
                         None if r["ok"] else int(r["raw_cq_status"]), "" if r["ok"] else r["status"])
        self._retained[h] = res
        while len(self._retained) > self.RETAINED:
            self._retained.pop(next(iter(self._retained)))
        return res

    def wait(self, io_handle: int, timeout_ms: int) -> tuple[str, str]:
        r = self.wait_result(io_handle, timeout_ms)
        return r.observation, r.state

    def wait_detail(self, io_handle: int, timeout_ms: int = 0) -> dict:
        return asdict(self.wait_result(io_handle, timeout_ms))

    def query_io(self, io_handle: int) -> str:
        h = int(io_handle)
        if h in self._retained:
            return self._retained[h].state
        return str(self.native.query_io(h)).upper()

    def release_io(self, io_handle: int) -> None:
        h = int(io_handle)
        if h not in self._retained:
            self.wait_result(h, 0)  # keep the terminal result readable after the release
        self.native.release_io(h)
        self._open.discard(h)

    def open_io_count(self) -> int:
        return len(self._open)

    def testing_force_complete(self, io_handle: int, state: str) -> None:
        """Stub runtimes only: make an in-flight IO terminal (``"COMPLETED"`` or ``"FAILED"``).

        A stub runtime's IO has no DataPath behind it and stays in flight until this
        call; a FAILED IO reports every accepted request as failed. Component-backed
        runtimes refuse (their DataPaths complete IO).
        """
        if state not in ("COMPLETED", "FAILED"):
            raise ValueError(f"state must be 'COMPLETED' or 'FAILED', got {state!r}")
        self.native.testing_force_complete(int(io_handle), state)

    def testing_inject_next_read_nvme_error(self, raw_cq_status: int) -> None:
        """The next command the first drive serves completes with ``raw_cq_status`` (type and code bits)."""
        if not hasattr(self.native, "inject"):
            raise ValueError("error injection needs a runtime with emulated NVMe controllers")
        self.native.inject(0, "media_error", 1, 0, int(raw_cq_status))

    def shutdown(self, timeout_ms: int) -> None:
        self.native.shutdown(int(timeout_ms))


OBJECT_STORE_SCHEMES = ("local_nvme_file", "striped_local_nvme_file")  # one mount / slots rotating over mounts
_STORE_KEYS = ("uri", "segment_bytes", "segment_count", "segment_file_slots", "segment_header_bytes",
               "capacity_slots", "capacity_bytes", "rank_id", "rank_count")


class ObjectStore:
    """Tutti's ``ObjectStore`` binding: ``open(scheme, config)`` with Tutti's config keys.

    ``devices`` is a list of ``{"mount_path": ...}`` (other device facts are
    accepted); ``namespace_fingerprint`` (bytes) guards the namespace's geometry.
    ``background_reclaim`` and ``residency_sync_interval_ms`` are accepted and
    have no effect here (residency bitmaps are memory-mapped and always current).
    """

    def __init__(self):
        self.native = None

    def open(self, scheme: str, config: dict) -> None:
        if self.native is not None:
            raise RuntimeError("object_store.open: store already open")
        if scheme not in OBJECT_STORE_SCHEMES:
            raise ValueError(f"unknown storage object store scheme {scheme!r} (one of {OBJECT_STORE_SCHEMES})")
        c = dict(config)
        mounts = [d["mount_path"] if isinstance(d, dict) else str(d) for d in c.get("devices") or []]
        if not mounts:
            raise ValueError("object store config needs devices (mount_path)")
        if scheme == "local_nvme_file" and len(mounts) != 1:
            raise ValueError("local_nvme_file takes exactly one device; striped_local_nvme_file takes several")
        ours = {k: c[k] for k in _STORE_KEYS if k in c}
        ours["mounts"] = mounts
        if c.get("namespace_fingerprint") is not None:
            ours["fingerprint"] = c["namespace_fingerprint"]
        store = _core().ObjectStore()
        store.open(ours)
        self.native = store

    def is_open(self) -> bool:
        return self.native is not None

    def close(self) -> None:
        if self.native is not None:
            store, self.native = self.native, None
            store.close()

    def _store(self):
        if self.native is None:
            raise RuntimeError("object store is not open")
        return self.native

    def contains_prefix(self, keys) -> int:
        return self._store().contains_prefix(list(keys), False)

    def contains_prefix_all_ranks(self, keys) -> int:
        return self._store().contains_prefix(list(keys), True)

    def ready_slots(self) -> int:
        return self._store().ready_slots

    def precreated_slots(self) -> int:
        return self._store().precreated_slots

    def precreate_target(self) -> int:
        return self._store().precreate_target

    def __getattr__(self, name):
        # contains, lookup, usage, reserve, commit, abort, release, pin, unpin, recover,
        # checkpoint, precreate_step, slot_uri, slot_generation: the same calls
        if name == "native":
            raise AttributeError(name)
        return getattr(self._store(), name)
