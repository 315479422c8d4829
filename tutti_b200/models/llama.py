"""Random-initialised Llama-3.x decoder with a paged KV pool, for prefill with
prefix reuse (the layerwise-overlap TTFT workload).

The pool uses the store's layout, ``pool[layer, plane, block, token, head, dim]``
(plane 0 = K, 1 = V). Prefill of ``new`` tokens for a request whose first
``cached`` tokens are already in the pool (restored by the store) writes the
new K/V into the request's next blocks and attends over all
``cached + new`` keys with a lower-right causal mask. A per-layer hook lets the
KV engine order each layer's attention after that layer's restore
(``wait_layer``) and kick off work after it (``after_layer``).

GEMMs are cuBLAS (torch.matmul); attention is PyTorch SDPA. These are the
model's compute, not the store's hot path.

Tensor parallelism (``tp_size`` > 1, one process per GPU): each rank holds
``heads / tp`` query heads, ``kv_heads / tp`` KV heads (or one KV head shared
by ``tp / kv_heads`` adjacent ranks when there are fewer KV heads than ranks),
``intermediate / tp`` MLP columns, and its slice of the paged pool; the
attention output and MLP down projections are row-parallel and their partial
sums are all-reduced over ``group`` (NCCL over NVLink on B200). Embedding and
LM head are replicated. ``full_init`` draws the unsharded weights and slices
them (identical to ``tp_size`` = 1; for tests); otherwise each rank draws its
own shards (random weights either way).
Parity: the reference drives the same pattern through vLLM's attention
backends and its connector hooks (tutti/integration/vllm/connector.py:370-374,
wait_for_layer_load / save_kv_layer); its C++ example
examples/layerwise_kv_overlap stands in a naive SGEMM for the model.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.nn.functional as F

from .kv_geometry import KVGeometry


@dataclass(frozen=True)
class LlamaConfig:
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5

    def kv_heads_per_rank(self, tp_size: int = 1) -> int:
        if self.kv_heads >= tp_size:
            if self.kv_heads % tp_size:
                raise ValueError(f"{self.kv_heads} KV heads do not split over TP{tp_size}")
            return self.kv_heads // tp_size
        if tp_size % self.kv_heads:
            raise ValueError(f"TP{tp_size} does not replicate {self.kv_heads} KV heads evenly")
        return 1

    def geometry(self, block_size: int = 16, chunk_tokens: int = 256, tp_size: int = 1) -> KVGeometry:
        """The KV geometry of one rank's slice (the whole model's at ``tp_size`` = 1)."""
        kv = self.kv_heads_per_rank(tp_size)
        name = f"llama-{self.layers}L-{self.kv_heads}kv" + (f"-tp{tp_size}" if tp_size > 1 else "")
        return KVGeometry(name, self.layers, kv, self.head_dim, block_size=block_size, chunk_tokens=chunk_tokens)


LLAMA_3_1_8B = LlamaConfig()
LLAMA_3_1_70B = LlamaConfig(hidden=8192, layers=80, heads=64, kv_heads=8, intermediate=28672)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class LlamaModel:
    """Weights as plain tensors (no nn.Module overhead); bf16 on one device (one TP rank's shards)."""

    def __init__(self, cfg: LlamaConfig, device: torch.device | str = "cuda", dtype=torch.bfloat16, seed: int = 0,
                 tp_rank: int = 0, tp_size: int = 1, group=None, full_init: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp_rank, self.tp_size, self.group = int(tp_rank), int(tp_size), group
        c = cfg
        if c.heads % tp_size or c.intermediate % tp_size:
            raise ValueError(f"{c.heads} heads / {c.intermediate} MLP columns do not split over TP{tp_size}")
        self.heads = c.heads // tp_size
        self.kv_heads = c.kv_heads_per_rank(tp_size)
        self.intermediate = c.intermediate // tp_size
        # first KV head of this rank (adjacent ranks share one when KV heads < TP)
        kv0 = tp_rank * self.kv_heads if c.kv_heads >= tp_size else tp_rank // (tp_size // c.kv_heads)
        D = c.head_dim
        g = torch.Generator(device=self.device).manual_seed(seed if full_init or tp_size == 1 else seed * 1009 + tp_rank)

        def w(*shape, scale=None):
            t = torch.empty(shape, device=self.device, dtype=dtype)
            std = scale if scale is not None else 1.0 / math.sqrt(shape[-1])
            return t.normal_(0.0, std, generator=g)

        def rows(full_rows, fan_in, pieces):
            """This rank's rows of a [full_rows, fan_in] weight: ``pieces`` = [(start, count), ...]."""
            if full_init:
                full = w(full_rows, fan_in)
                return torch.cat([full[a:a + n] for a, n in pieces])
            return w(sum(n for _, n in pieces), fan_in)

        def cols(fan_out, full_cols, start, count):
            if full_init:
                return w(fan_out, full_cols)[:, start:start + count].contiguous()
            t = w(fan_out, count, scale=1.0 / math.sqrt(full_cols))
            return t

        q_out, kv_out = c.heads * D, c.kv_heads * D
        self.embed = w(c.vocab, c.hidden, scale=0.02)
        self.layers = []
        for _ in range(c.layers):
            qkv_pieces = [(tp_rank * self.heads * D, self.heads * D),
                          (q_out + kv0 * D, self.kv_heads * D),
                          (q_out + kv_out + kv0 * D, self.kv_heads * D)]
            mlp_pieces = [(tp_rank * self.intermediate, self.intermediate),
                          (c.intermediate + tp_rank * self.intermediate, self.intermediate)]
            self.layers.append({
                "ln1": torch.ones(c.hidden, device=self.device, dtype=dtype),
                "wqkv": rows(q_out + 2 * kv_out, c.hidden, qkv_pieces),
                "wo": cols(c.hidden, q_out, tp_rank * self.heads * D, self.heads * D),
                "ln2": torch.ones(c.hidden, device=self.device, dtype=dtype),
                "w13": rows(2 * c.intermediate, c.hidden, mlp_pieces),
                "w2": cols(c.hidden, c.intermediate, tp_rank * self.intermediate, self.intermediate),
            })
        self.norm = torch.ones(c.hidden, device=self.device, dtype=dtype)
        self.lm_head = w(c.vocab, c.hidden, scale=0.02)
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=self.device, dtype=torch.float32)
                                        / c.head_dim))
        self._inv_freq = inv

    def _reduce(self, partial: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel GEMM's partial outputs over the TP group (in place)."""
        if self.tp_size > 1:
            import torch.distributed as dist

            dist.all_reduce(partial, group=self.group)
        return partial

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        # x [T, H, D], pos [T]
        f = pos.float()[:, None] * self._inv_freq[None, :]
        cos, sin = f.cos()[:, None, :], f.sin()[:, None, :]
        x1, x2 = x[..., ::2].float(), x[..., 1::2].float()
        out = torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2)
        return out.to(x.dtype)

    @torch.inference_mode()
    def prefill(self, tokens: Sequence[torch.Tensor], cached: Sequence[int], block_tables: Sequence[torch.Tensor],
                pool: torch.Tensor, *, wait_layer: Callable[[int], None] | None = None,
                after_layer: Callable[[int], None] | None = None) -> torch.Tensor:
        """Prefill ``tokens[r]`` (new tokens) after ``cached[r]`` reused tokens.

        ``block_tables[r]`` lists the pool blocks of request r covering
        ``cached[r] + len(tokens[r])`` tokens. Returns last-token logits [R, vocab].
        """
        c = self.cfg
        H, KV, I = self.heads, self.kv_heads, self.intermediate
        bs = pool.shape[3]
        R = len(tokens)
        lens = [int(t.numel()) for t in tokens]
        x = self.embed[torch.cat([t.to(self.device) for t in tokens])]
        pos = torch.cat([torch.arange(cached[r], cached[r] + lens[r], device=self.device) for r in range(R)])
        # destination slots of the new tokens: (block, offset) per token
        slot_block, slot_off = [], []
        for r in range(R):
            p = torch.arange(cached[r], cached[r] + lens[r], device=self.device)
            bt = block_tables[r].to(self.device)
            slot_block.append(bt[p // bs])
            slot_off.append(p % bs)
        slot_block = torch.cat(slot_block)
        slot_off = torch.cat(slot_off)
        q_out = H * c.head_dim
        kv_out = KV * c.head_dim
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        for li, L in enumerate(self.layers):
            h = _rms(x, L["ln1"], c.rms_eps)
            qkv = h @ L["wqkv"].t()
            q = qkv[:, :q_out].view(-1, H, c.head_dim)
            k = qkv[:, q_out:q_out + kv_out].view(-1, KV, c.head_dim)
            v = qkv[:, q_out + kv_out:].view(-1, KV, c.head_dim)
            q = self._rope(q, pos)
            k = self._rope(k, pos)
            if wait_layer is not None:
                wait_layer(li)  # the restored prefix of this layer must be in the pool
            pool[li, 0, slot_block, slot_off] = k
            pool[li, 1, slot_block, slot_off] = v
            outs = []
            for r in range(R):
                total = cached[r] + lens[r]
                nblk = (total + bs - 1) // bs
                bt = block_tables[r][:nblk].to(self.device)
                kk = pool[li, 0, bt].reshape(-1, KV, c.head_dim)[:total]
                vv = pool[li, 1, bt].reshape(-1, KV, c.head_dim)[:total]
                qr = q[starts[r]:starts[r + 1]].transpose(0, 1).unsqueeze(0)  # [1, H, Tq, D]
                kr = kk.transpose(0, 1).unsqueeze(0)
                vr = vv.transpose(0, 1).unsqueeze(0)
                from torch.nn.attention.bias import causal_lower_right

                o = F.scaled_dot_product_attention(qr, kr, vr, attn_mask=causal_lower_right(qr.shape[2], kr.shape[2]),
                                                   enable_gqa=True)
                outs.append(o.squeeze(0).transpose(0, 1).reshape(-1, q_out))
            if after_layer is not None:
                after_layer(li)
            x = x + self._reduce(torch.cat(outs) @ L["wo"].t())
            h = _rms(x, L["ln2"], c.rms_eps)
            gu = h @ L["w13"].t()
            gate, up = gu[:, :I], gu[:, I:]
            x = x + self._reduce((F.silu(gate) * up) @ L["w2"].t())
        last = torch.tensor([s - 1 for s in starts[1:]], device=self.device)
        return _rms(x[last], self.norm, c.rms_eps) @ self.lm_head.t()
