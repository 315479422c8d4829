"""Synchronous vs asynchronous load decision.

A synchronous load runs layerwise inside the request's first forward (its
restore overlaps the prefill); an asynchronous load parks the request in
WAITING_FOR_REMOTE_KVS while other requests compute. Long loads that would
stall the batch for longer than ``max_sync_stall_ms`` go asynchronous. The
estimate uses EWMAs of the measured restore bandwidth.
Parity: reference tutti/integration/vllm/load_policy.py:54-172 (EWMA policy,
modes sync|async|auto).
"""
from __future__ import annotations


class LoadPolicy:
    def __init__(self, mode: str = "sync", bytes_per_token: int = 131072, max_sync_stall_ms: float = 500.0,
                 initial_gbps: float = 30.0, alpha: float = 0.2):
        if mode not in ("sync", "async", "auto"):
            raise ValueError("load mode must be sync, async or auto")
        self.mode = mode
        self.bytes_per_token = bytes_per_token
        self.max_sync_stall_ms = max_sync_stall_ms
        self.gbps = initial_gbps
        self.alpha = alpha

    def observe(self, nbytes: int, seconds: float) -> None:
        if seconds > 0 and nbytes > 0:
            self.gbps = (1 - self.alpha) * self.gbps + self.alpha * (nbytes / seconds / 1e9)

    def estimate_ms(self, tokens: int) -> float:
        return tokens * self.bytes_per_token / (self.gbps * 1e9) * 1e3

    def choose_async(self, tokens: int) -> bool:
        if self.mode == "sync":
            return False
        if self.mode == "async":
            return True
        return self.estimate_ms(tokens) > self.max_sync_stall_ms
