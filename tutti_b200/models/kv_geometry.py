"""KV-cache geometries of the model families the store serves.

A geometry says how one layer's KV for one block of tokens is laid out in
the engine's paged pool and how many bytes a chunk occupies on disk. The
reference derives the same facts from vLLM's KVCacheConfig
(tutti/integration/vllm/geometry.py) and its per-entity page geometry for
MiniMax main-KV plus index caches (tutti/storage/tutti_nvme/layerwise_direct.py:18-181).

Pool layout used by this package (vLLM FlashAttention layout, one tensor for
all layers):  pool[layer, plane, block, token_in_block, head, dim] with
plane 0 = K, 1 = V (``planes=2``) or a single latent plane for MLA
(``planes=1``). A block's bytes for one (layer, plane) are contiguous.
On disk, one chunk of ``chunk_tokens`` tokens is one object; segment l holds
layer l: for each block j of the chunk, plane 0 then plane 1.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class KVGeometry:
    name: str
    num_layers: int
    num_kv_heads: int
    head_dim: int
    block_size: int = 16
    planes: int = 2  # K and V; 1 for MLA latent caches
    dtype: torch.dtype = torch.bfloat16
    chunk_tokens: int = 256
    tp_size: int = 1

    @property
    def elem_bytes(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    @property
    def heads_per_rank(self) -> int:
        assert self.num_kv_heads % self.tp_size == 0 or self.num_kv_heads < self.tp_size
        return max(1, self.num_kv_heads // self.tp_size)

    @property
    def plane_block_bytes(self) -> int:
        """Bytes of one (layer, plane, block) in the pool of one rank."""
        return self.block_size * self.heads_per_rank * self.head_dim * self.elem_bytes

    @property
    def block_layer_bytes(self) -> int:
        return self.planes * self.plane_block_bytes

    @property
    def blocks_per_chunk(self) -> int:
        assert self.chunk_tokens % self.block_size == 0
        return self.chunk_tokens // self.block_size

    @property
    def segment_bytes(self) -> int:
        """On-disk bytes of one layer of one chunk (rank-local slice)."""
        return self.blocks_per_chunk * self.block_layer_bytes

    @property
    def chunk_bytes(self) -> int:
        return self.num_layers * self.segment_bytes

    def pool_shape(self, num_blocks: int) -> tuple[int, ...]:
        return (self.num_layers, self.planes, num_blocks, self.block_size, self.heads_per_rank, self.head_dim)

    def pool_bytes(self, num_blocks: int) -> int:
        return self.num_layers * self.planes * num_blocks * self.plane_block_bytes

    def prefix_bytes(self, tokens: int) -> int:
        return (tokens // self.block_size) * self.num_layers * self.block_layer_bytes

    def with_tp(self, tp: int) -> "KVGeometry":
        return KVGeometry(self.name, self.num_layers, self.num_kv_heads, self.head_dim, self.block_size,
                          self.planes, self.dtype, self.chunk_tokens, tp)

    def fingerprint(self) -> str:
        return (f"{self.name}:L{self.num_layers}:H{self.heads_per_rank}/{self.num_kv_heads}:D{self.head_dim}"
                f":B{self.block_size}:P{self.planes}:{str(self.dtype).split('.')[-1]}:C{self.chunk_tokens}"
                f":TP{self.tp_size}")


LLAMA3_8B = KVGeometry("llama-3.1-8b", num_layers=32, num_kv_heads=8, head_dim=128)
LLAMA3_70B = KVGeometry("llama-3.1-70b", num_layers=80, num_kv_heads=8, head_dim=128)
# DeepSeek-V3 MLA latent cache: 512 latent + 64 RoPE values per token, one plane.
DEEPSEEK_V3_MLA = KVGeometry("deepseek-v3-mla", num_layers=61, num_kv_heads=1, head_dim=576,
                             block_size=64, planes=1, chunk_tokens=256)
# DeepSeek-V3.2-style indexer cache: 128 fp8 values + one fp32 scale per token.
DEEPSEEK_V3_INDEXER = KVGeometry("deepseek-v3-indexer", num_layers=61, num_kv_heads=1, head_dim=132,
                                 block_size=64, planes=1, dtype=torch.uint8, chunk_tokens=256)

GEOMETRIES = {g.name: g for g in (LLAMA3_8B, LLAMA3_70B, DEEPSEEK_V3_MLA, DEEPSEEK_V3_INDEXER)}
