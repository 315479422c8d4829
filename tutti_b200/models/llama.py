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

    def geometry(self, block_size: int = 16, chunk_tokens: int = 256) -> KVGeometry:
        return KVGeometry(f"llama-{self.layers}L-{self.kv_heads}kv", self.layers, self.kv_heads, self.head_dim,
                          block_size=block_size, chunk_tokens=chunk_tokens)


LLAMA_3_1_8B = LlamaConfig()
LLAMA_3_1_70B = LlamaConfig(hidden=8192, layers=80, heads=64, kv_heads=8, intermediate=28672)


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


class LlamaModel:
    """Weights as plain tensors (no nn.Module overhead); bf16 on one device."""

    def __init__(self, cfg: LlamaConfig, device: torch.device | str = "cuda", dtype=torch.bfloat16, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        g = torch.Generator(device=self.device).manual_seed(seed)

        def w(*shape, scale=None):
            t = torch.empty(shape, device=self.device, dtype=dtype)
            std = scale if scale is not None else 1.0 / math.sqrt(shape[-1])
            return t.normal_(0.0, std, generator=g)

        c = cfg
        q_out = c.heads * c.head_dim
        kv_out = c.kv_heads * c.head_dim
        self.embed = w(c.vocab, c.hidden, scale=0.02)
        self.layers = []
        for _ in range(c.layers):
            self.layers.append({
                "ln1": torch.ones(c.hidden, device=self.device, dtype=dtype),
                "wqkv": w(q_out + 2 * kv_out, c.hidden),
                "wo": w(c.hidden, q_out),
                "ln2": torch.ones(c.hidden, device=self.device, dtype=dtype),
                "w13": w(2 * c.intermediate, c.hidden),
                "w2": w(c.hidden, c.intermediate),
            })
        self.norm = torch.ones(c.hidden, device=self.device, dtype=dtype)
        self.lm_head = w(c.vocab, c.hidden, scale=0.02)
        inv = 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, device=self.device, dtype=torch.float32)
                                        / c.head_dim))
        self._inv_freq = inv

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
        q_out = c.heads * c.head_dim
        kv_out = c.kv_heads * c.head_dim
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        for li, L in enumerate(self.layers):
            h = _rms(x, L["ln1"], c.rms_eps)
            qkv = h @ L["wqkv"].t()
            q = qkv[:, :q_out].view(-1, c.heads, c.head_dim)
            k = qkv[:, q_out:q_out + kv_out].view(-1, c.kv_heads, c.head_dim)
            v = qkv[:, q_out + kv_out:].view(-1, c.kv_heads, c.head_dim)
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
                kk = pool[li, 0, bt].reshape(-1, c.kv_heads, c.head_dim)[:total]
                vv = pool[li, 1, bt].reshape(-1, c.kv_heads, c.head_dim)[:total]
                qr = q[starts[r]:starts[r + 1]].transpose(0, 1).unsqueeze(0)  # [1, H, Tq, D]
                kr = kk.transpose(0, 1).unsqueeze(0)
                vr = vv.transpose(0, 1).unsqueeze(0)
                from torch.nn.attention.bias import causal_lower_right

                o = F.scaled_dot_product_attention(qr, kr, vr, attn_mask=causal_lower_right(qr.shape[2], kr.shape[2]),
                                                   enable_gqa=True)
                outs.append(o.squeeze(0).transpose(0, 1).reshape(-1, q_out))
            if after_layer is not None:
                after_layer(li)
            x = x + torch.cat(outs) @ L["wo"].t()
            h = _rms(x, L["ln2"], c.rms_eps)
            gu = h @ L["w13"].t()
            gate, up = gu[:, :c.intermediate], gu[:, c.intermediate:]
            x = x + (F.silu(gate) * up) @ L["w2"].t()
        last = torch.tensor([s - 1 for s in starts[1:]], device=self.device)
        return _rms(x[last], self.norm, c.rms_eps) @ self.lm_head.t()
