"""Tensor-parallel Llama prefill (gloo ranks on CPU, float32): every rank's logits equal the
unsharded model's, with the prefix restored in the pool and with fewer KV heads than ranks."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tutti_b200.models.llama import LlamaConfig, LlamaModel

SMALL = LlamaConfig(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, intermediate=96, vocab=97)
ONE_KV = LlamaConfig(hidden=64, layers=2, heads=4, kv_heads=1, head_dim=16, intermediate=96, vocab=97)
BS = 4


def _inputs(cfg):
    g = torch.Generator().manual_seed(3)
    toks = [torch.randint(0, cfg.vocab, (9,), generator=g), torch.randint(0, cfg.vocab, (5,), generator=g)]
    tables = [torch.tensor([0, 1, 2, 3]), torch.tensor([5, 6, 7])]
    return toks, tables


def _run(cfg, rank, world, group, cached_prefix: bool):
    model = LlamaModel(cfg, "cpu", dtype=torch.float32, seed=11, tp_rank=rank, tp_size=world, group=group,
                       full_init=True)
    kv = cfg.kv_heads_per_rank(world)
    pool = torch.zeros(cfg.layers, 2, 8, BS, kv, cfg.head_dim)
    toks, tables = _inputs(cfg)
    if not cached_prefix:
        return model.prefill(toks, [0, 0], tables, pool), pool
    # prefill the first 4 tokens of each request, then the rest after that cached prefix
    model.prefill([t[:4] for t in toks], [0, 0], tables, pool)
    return model.prefill([t[4:] for t in toks], [4, 4], tables, pool), pool


def _rank(rank, world, port, q, cfg_name, cached):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = {"small": SMALL, "one_kv": ONE_KV}[cfg_name]
        logits, pool = _run(cfg, rank, world, dist.group.WORLD, cached)
        q.put((rank, (logits.numpy(), pool.numpy())))  # by value: the rank exits after this
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, "".join(traceback.format_exception(e))[-2000:]))
    finally:
        dist.destroy_process_group()


def _spawn(world, *args):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, world, port, q, *args)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=30)
    return out


@pytest.mark.parametrize("cfg_name,cached", [("small", False), ("small", True), ("one_kv", True)])
def test_tp2_prefill_matches_the_unsharded_model(cfg_name, cached):
    cfg = {"small": SMALL, "one_kv": ONE_KV}[cfg_name]
    ref_logits, ref_pool = _run(cfg, 0, 1, None, cached)
    out = _spawn(2, cfg_name, cached)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
        logits, pool = (torch.from_numpy(a) for a in out[r])
        torch.testing.assert_close(logits, ref_logits, rtol=1e-4, atol=1e-4)
        # rank r's pool holds its KV heads of the reference pool
        if cfg.kv_heads >= 2:
            want = ref_pool[..., r * (cfg.kv_heads // 2):(r + 1) * (cfg.kv_heads // 2), :]
        else:
            want = ref_pool  # one KV head, held by both ranks
        torch.testing.assert_close(pool, want, rtol=1e-4, atol=1e-4)


def test_tp_geometry_and_shapes():
    assert SMALL.geometry(tp_size=2).num_kv_heads == 1 and ONE_KV.geometry(tp_size=2).num_kv_heads == 1
    with pytest.raises(ValueError):
        LlamaConfig(kv_heads=8).kv_heads_per_rank(3)
    with pytest.raises(ValueError):
        LlamaModel(SMALL, "cpu", torch.float32, tp_size=3)
    m = LlamaModel(SMALL, "cpu", torch.float32, tp_rank=1, tp_size=2)
    L = m.layers[0]
    assert L["wqkv"].shape == (2 * 16 + 2 * 16, 64) and L["wo"].shape == (64, 32)
    assert L["w13"].shape == (96, 64) and L["w2"].shape == (64, 48)
