"""Torch-facing wrappers of the sm_100a kernels in ``tutti_b200._ops``.

* ``page_copy`` / ``gather_blocks`` / ``scatter_blocks``: the staged paged
  transfer (pool blocks <-> a contiguous staging buffer laid out like the
  on-disk chunk segment) and peer page pulls, one batched bulk-copy kernel.
  Parity: reference csrc/kv_transfer/src/mem_kernels.cu (single_layer_kv_transfer,
  replica_page_scatter).
* ``fp8_quant`` / ``fp8_dequant`` and the paged ``fp8_gather_quant`` /
  ``fp8_dequant_scatter``: E4M3 with one fp32 scale per 1x128 group.
* ``prefix_hash``: chained BLAKE2b-128 chunk keys computed on the GPU,
  bit-identical to ``tutti_b200.index.chunk_index.chunk_keys_for_tokens``.
* ``kv_checksum``: 64-bit order-sensitive digests of pool blocks.
"""
from __future__ import annotations

from typing import Sequence

import torch

from .._native import ops as _ops
from ..index.chunk_index import KEY_BYTES, chunk_digest


def _items(src_ptrs: torch.Tensor, dst_ptrs: torch.Tensor, sizes: torch.Tensor | int) -> torch.Tensor:
    n = src_ptrs.numel()
    if isinstance(sizes, int):
        sizes = torch.full((n,), sizes, dtype=torch.int64, device=src_ptrs.device)
    return torch.stack([src_ptrs.reshape(-1), dst_ptrs.reshape(-1), sizes.reshape(-1)], dim=1).contiguous()


def page_copy(src_ptrs: torch.Tensor, dst_ptrs: torch.Tensor, sizes: torch.Tensor | int, *, tma: bool = True) -> None:
    """Copy ``sizes[i]`` bytes from address ``src_ptrs[i]`` to ``dst_ptrs[i]`` (int64 CUDA tensors).

    Addresses and sizes must be multiples of 16. ``tma=False`` selects the
    vector-load path, required when either side is another GPU's memory.
    """
    if src_ptrs.numel() == 0:
        return
    _ops().copy_items(_items(src_ptrs, dst_ptrs, sizes), tma)


def _block_ptrs(pool: torch.Tensor, block_ids: torch.Tensor, layers: torch.Tensor) -> torch.Tensor:
    """Addresses of pool[l, p, b] in (block, layer, plane) order -> [nb, L, P]."""
    L, P, NB = pool.shape[0], pool.shape[1], pool.shape[2]
    plane_bytes = pool[0, 0, 0].numel() * pool.element_size()
    b = block_ids.to(pool.device, torch.int64).reshape(-1, 1, 1)
    lay = layers.to(pool.device, torch.int64).reshape(1, -1, 1)
    p = torch.arange(P, device=pool.device, dtype=torch.int64).reshape(1, 1, -1)
    return pool.data_ptr() + ((lay * P + p) * NB + b) * plane_bytes


def _staging_ptrs(staging: torch.Tensor, nb: int, nl: int, P: int, plane_bytes: int, blocks_per_chunk: int):
    """Staging layout of chunk segments: [chunk][layer][block_in_chunk][plane] -> [nb, L, P] addresses."""
    j = torch.arange(nb, device=staging.device, dtype=torch.int64)
    chunk, jb = j // blocks_per_chunk, j % blocks_per_chunk
    lay = torch.arange(nl, device=staging.device, dtype=torch.int64)
    p = torch.arange(P, device=staging.device, dtype=torch.int64)
    seg = blocks_per_chunk * P * plane_bytes
    off = (chunk.reshape(-1, 1, 1) * nl * seg + lay.reshape(1, -1, 1) * seg
           + jb.reshape(-1, 1, 1) * P * plane_bytes + p.reshape(1, 1, -1) * plane_bytes)
    return staging.data_ptr() + off


def gather_blocks(pool: torch.Tensor, block_ids: torch.Tensor, blocks_per_chunk: int,
                  layers: Sequence[int] | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Pool blocks -> contiguous chunk segments (the staged store path)."""
    L, P = pool.shape[0], pool.shape[1]
    layers_t = torch.arange(L) if layers is None else torch.as_tensor(list(layers))
    nb = block_ids.numel()
    plane_bytes = pool[0, 0, 0].numel() * pool.element_size()
    nbytes = nb * layers_t.numel() * P * plane_bytes
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=pool.device)
    src = _block_ptrs(pool, block_ids, layers_t)
    dst = _staging_ptrs(out, nb, layers_t.numel(), P, plane_bytes, blocks_per_chunk)
    page_copy(src, dst, plane_bytes)
    return out


def scatter_blocks(staging: torch.Tensor, pool: torch.Tensor, block_ids: torch.Tensor, blocks_per_chunk: int,
                   layers: Sequence[int] | None = None) -> None:
    """Contiguous chunk segments -> pool blocks (the staged restore path)."""
    L, P = pool.shape[0], pool.shape[1]
    layers_t = torch.arange(L) if layers is None else torch.as_tensor(list(layers))
    nb = block_ids.numel()
    plane_bytes = pool[0, 0, 0].numel() * pool.element_size()
    src = _staging_ptrs(staging, nb, layers_t.numel(), P, plane_bytes, blocks_per_chunk)
    dst = _block_ptrs(pool, block_ids, layers_t)
    page_copy(src, dst, plane_bytes)


def fp8_quant(x: torch.Tensor, group: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """x [rows, cols] -> (fp8 E4M3 bytes [rows, cols] as uint8, fp32 scales [rows, cols/128])."""
    return _ops().fp8_quant(x.contiguous(), group)


def fp8_dequant(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    return _ops().fp8_dequant(q.contiguous(), scale.contiguous(), dtype)


def fp8_gather_quant(pool: torch.Tensor, row_offsets: torch.Tensor, cols: int):
    """Quantise bf16 rows found at byte offsets of ``pool`` (fused paged gather)."""
    return _ops().fp8_gather_quant(pool, row_offsets.to(torch.int64).contiguous(), cols)


def fp8_dequant_scatter(q: torch.Tensor, scale: torch.Tensor, pool: torch.Tensor, row_offsets: torch.Tensor) -> None:
    """Dequantise into bf16 rows at byte offsets of ``pool`` (fused paged scatter)."""
    _ops().fp8_dequant_scatter(q.contiguous(), scale.contiguous(), pool, row_offsets.to(torch.int64).contiguous())


def prefix_hash(requests: Sequence[Sequence[int]] | Sequence[torch.Tensor], chunk_tokens: int,
                namespace: bytes = b"", device: torch.device | str = "cuda") -> list[list[bytes]]:
    """Chained chunk keys of each request's tokens, computed on the GPU.

    A namespace that is neither empty nor 16 bytes is folded into the first
    key on the host (it is not a whole number of 8-byte words).
    """
    dev = torch.device(device)
    toks, starts, lengths, parents, plen, koff = [], [], [], [], [], []
    pos = 0
    keys_before = 0
    first_keys: list[bytes | None] = []
    for r in requests:
        t = r.to("cpu", torch.int64) if isinstance(r, torch.Tensor) else torch.as_tensor(list(r), dtype=torch.int64)
        first = None
        if namespace and len(namespace) != KEY_BYTES and t.numel() >= chunk_tokens:
            first = chunk_digest(namespace, t[:chunk_tokens].tolist())
            t = t[chunk_tokens:]
            parents.append(torch.frombuffer(bytearray(first), dtype=torch.uint8))
            plen.append(16)
        elif len(namespace) == KEY_BYTES:
            parents.append(torch.frombuffer(bytearray(namespace), dtype=torch.uint8))
            plen.append(16)
        else:
            parents.append(torch.zeros(16, dtype=torch.uint8))
            plen.append(0)
        first_keys.append(first)
        n = t.numel() // chunk_tokens
        toks.append(t)
        starts.append(pos)
        lengths.append(t.numel())
        koff.append(keys_before)
        pos += t.numel()
        keys_before += n
    if not toks:
        return []
    tok = torch.cat(toks).to(dev)
    out = _ops().prefix_hash(tok, torch.tensor(starts, device=dev), torch.tensor(lengths, device=dev),
                             torch.stack(parents).to(dev), torch.tensor(plen, dtype=torch.int32, device=dev),
                             torch.tensor(koff, device=dev), max(keys_before, 1), chunk_tokens)
    raw = out.cpu().numpy().tobytes()
    result = []
    for i, (k0, n) in enumerate(zip(koff, [ln // chunk_tokens for ln in lengths])):
        ks = [raw[16 * (k0 + c): 16 * (k0 + c + 1)] for c in range(n)]
        if first_keys[i] is not None:
            ks = [first_keys[i]] + ks
        result.append(ks)
    return result


def kv_checksum(pool: torch.Tensor, block_ids: torch.Tensor, layers: Sequence[int] | None = None) -> torch.Tensor:
    """int64 digests [nb, L, P] of pool[l, p, b] for the given blocks."""
    L, P = pool.shape[0], pool.shape[1]
    layers_t = torch.arange(L) if layers is None else torch.as_tensor(list(layers))
    plane_bytes = pool[0, 0, 0].numel() * pool.element_size()
    ptrs = _block_ptrs(pool, block_ids, layers_t)
    items = _items(ptrs, torch.zeros_like(ptrs), plane_bytes)
    # every item is one plane page: the segment-parallel kernel applies when pages are 16-byte multiples
    return _ops().checksum(items, plane_bytes if plane_bytes % 16 == 0 else 0).reshape(ptrs.shape)


def ipc_export(t: torch.Tensor):
    return _ops().ipc_export(t)


def ipc_open(handle: bytes, device: int) -> int:
    return _ops().ipc_open(handle, device)


def ipc_close(ptr: int, device: int) -> None:
    _ops().ipc_close(ptr, device)


def enable_peer_access(device: int, peer: int) -> bool:
    return _ops().enable_peer_access(device, peer)


def ready_signal(targets: torch.Tensor, value: int) -> None:
    """Store ``value`` into every word whose address is in ``targets`` (int64 CUDA tensor), on the
    current stream, after the stream's earlier work (system-scope fence, release stores)."""
    _ops().ready_signal(targets, int(value))


def ready_wait(words: int, n: int, value: int, timeout_ns: int, status: torch.Tensor) -> None:
    """Make the current stream wait until the ``n`` 64-bit words at device address ``words`` all hold
    at least ``value``, for at most ``timeout_ns``; ``status[0]`` becomes 0, or a mask of the words
    still below ``value`` when the deadline passed (the stream then continues)."""
    _ops().ready_wait(int(words), int(n), int(value), int(timeout_ns), status)
