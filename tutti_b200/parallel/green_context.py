"""An IO stream confined to a few SMs (a CUDA green context), opt-in.

Persistent GEMM kernels hold every SM; an io kernel launched beside them
either waits for a whole wave or pushes them into a second one. A green
context splits the GPU's SMs: the io kernels run on a stream of a small SM
partition and the model keeps the rest. Enable it with
``TUTTI_GREEN_CTX_IO_SMS=<n>`` (the KV engine then creates its IO stream here)
or call ``io_stream_on_sms`` directly; keep the data path's ``max_ctas_per_op``
at or below the partition's SM count, since the io kernel runs one CTA per SM.
Parity: reference tutti/integration/vllm/green_context.py:33-66
(TUTTI_GREEN_CTX_IO_SMS) and doc/design/kv-storage-layout-and-io-submission.md
(inter-kernel gap p50 2.5-2.8 ms -> 19 us with 8 IO SMs).
"""
from __future__ import annotations

import os

import torch

ENV = "TUTTI_GREEN_CTX_IO_SMS"


def _check(res, what: str):
    err = res[0] if isinstance(res, tuple) else res
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: CUresult {int(err)}")
    if isinstance(res, tuple):
        return res[1] if len(res) == 2 else res[1:]
    return None


class GreenIoStream:
    """A green context of ``sms`` SMs on ``device`` and a non-blocking stream in it."""

    def __init__(self, sms: int, device: int = 0):
        from cuda.bindings import driver as d

        self._d = d
        torch.cuda.init()
        _check(d.cuInit(0), "cuInit")
        dev = _check(d.cuDeviceGet(int(device)), "cuDeviceGet")
        res = _check(d.cuDeviceGetDevResource(dev, d.CUdevResourceType.CU_DEV_RESOURCE_TYPE_SM),
                     "cuDeviceGetDevResource")
        total = int(res.sm.smCount)
        want = max(8, (int(sms) + 7) // 8 * 8)  # partitions are granted in groups of SMs
        if want >= total:
            raise ValueError(f"asked for {sms} IO SMs of {total}")
        out = _check(d.cuDevSmResourceSplitByCount(1, res, 0, want), "cuDevSmResourceSplitByCount")
        groups = out[0]
        part = groups[0] if isinstance(groups, (list, tuple)) else groups
        desc = _check(d.cuDevResourceGenerateDesc([part], 1), "cuDevResourceGenerateDesc")
        self.ctx = _check(d.cuGreenCtxCreate(desc, dev, d.CUgreenCtxCreate_flags.CU_GREEN_CTX_DEFAULT_STREAM),
                          "cuGreenCtxCreate")
        raw = _check(d.cuGreenCtxStreamCreate(self.ctx, d.CUstream_flags.CU_STREAM_NON_BLOCKING, 0),
                     "cuGreenCtxStreamCreate")
        self._raw = raw
        self.sms = int(part.sm.smCount)
        self.device = int(device)
        self.stream = torch.cuda.ExternalStream(int(raw), device=torch.device("cuda", self.device))

    def close(self) -> None:
        d = self._d
        if getattr(self, "_raw", None) is not None:
            d.cuStreamDestroy(self._raw)
            self._raw = None
        if getattr(self, "ctx", None) is not None:
            d.cuGreenCtxDestroy(self.ctx)
            self.ctx = None


_streams: dict[int, GreenIoStream] = {}


def io_stream_on_sms(sms: int, device: int = 0) -> torch.cuda.Stream:
    """The process's IO stream confined to ``sms`` SMs of ``device`` (created once per device)."""
    g = _streams.get(device)
    if g is None:
        g = GreenIoStream(sms, device)
        _streams[device] = g
    return g.stream


def configured_io_sms() -> int:
    v = os.environ.get(ENV, "").strip()
    return int(v) if v else 0
