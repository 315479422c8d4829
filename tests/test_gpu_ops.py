"""sm_100a ops against plain PyTorch / hashlib references."""
import numpy as np
import pytest
import torch

from tutti_b200 import ops
from tutti_b200.index.chunk_index import chunk_keys_for_tokens

pytestmark = pytest.mark.gpu


def test_page_copy_tma_and_simt_exact():
    src = torch.randint(0, 255, (1 << 22,), dtype=torch.uint8, device="cuda")
    for tma in (True, False):
        dst = torch.zeros_like(src)
        n = 97
        sizes = (torch.randint(1, 2048, (n,), device="cuda") * 16).to(torch.int64)
        offs = torch.cumsum(sizes, 0) - sizes
        # destinations: the same items laid out in a permuted order (no overlap)
        perm = torch.randperm(n, device="cuda")
        dsz = sizes[perm]
        doffs = torch.empty_like(offs)
        doffs[perm] = torch.cumsum(dsz, 0) - dsz
        ops.page_copy(src.data_ptr() + offs, dst.data_ptr() + doffs, sizes, tma=tma)
        torch.cuda.synchronize()
        for i in range(0, n, 7):
            a, b, s = int(offs[i]), int(doffs[i]), int(sizes[i])
            assert torch.equal(dst[b:b + s], src[a:a + s])


def test_gather_scatter_blocks_roundtrip():
    L, P, NB, bs, H, D = 4, 2, 64, 16, 8, 128
    pool = torch.randn(L, P, NB, bs, H, D, dtype=torch.bfloat16, device="cuda")
    blocks = torch.randperm(NB, device="cuda")[:16]
    staging = ops.gather_blocks(pool, blocks, blocks_per_chunk=4)
    # reference: chunk segments [chunk][layer][block][plane]
    ref = pool[:, :, blocks].permute(2, 0, 1, 3, 4, 5).reshape(4, 4, L, P, bs, H, D).permute(0, 2, 1, 3, 4, 5, 6)
    assert torch.equal(staging.view(torch.bfloat16).reshape(ref.shape), ref.contiguous())
    out = torch.zeros_like(pool)
    dst = torch.randperm(NB, device="cuda")[:16]
    ops.scatter_blocks(staging, out, dst, blocks_per_chunk=4)
    assert torch.equal(out[:, :, dst], pool[:, :, blocks])


def fp8_reference(x: torch.Tensor):
    g = x.float().reshape(x.shape[0], -1, 128)
    amax = g.abs().amax(dim=-1, keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (g / scale).to(torch.float8_e4m3fn)
    return q.reshape(x.shape), scale.squeeze(-1)


def test_fp8_quant_dequant_matches_fp32_reference():
    x = torch.randn(4096, 512, device="cuda", dtype=torch.bfloat16) * 3
    q, s = ops.fp8_quant(x)
    rq, rs = fp8_reference(x)
    torch.testing.assert_close(s, rs, rtol=1e-6, atol=0)
    mism = (q != rq.view(torch.uint8)).float().mean().item()
    assert mism < 1e-3  # only x*(1/s) vs x/s rounding ties may differ
    deq = ops.fp8_dequant(q, s, torch.float32)
    ref = (rq.float().reshape(4096, 4, 128) * rs.unsqueeze(-1)).reshape(4096, 512)
    err = (deq - x.float()).abs().reshape(4096, 4, 128).amax(-1)
    assert torch.all(err <= 0.0625 * x.float().abs().reshape(4096, 4, 128).amax(-1) + 1e-6)
    same = q == rq.view(torch.uint8)
    torch.testing.assert_close(deq[same], ref[same], rtol=1e-6, atol=1e-6)


def test_fp8_paged_gather_quant_and_dequant_scatter():
    pool = torch.randn(256, 128, dtype=torch.bfloat16, device="cuda")
    rows = torch.randperm(256, device="cuda")[:64]
    offs = rows * 128 * 2
    q, s = ops.fp8_gather_quant(pool.view(torch.uint8), offs, 128)
    q2, s2 = ops.fp8_quant(pool[rows])
    assert torch.equal(q, q2) and torch.equal(s, s2)
    out = torch.zeros_like(pool)
    dst = torch.randperm(256, device="cuda")[:64]
    ops.fp8_dequant_scatter(q, s, out.view(torch.uint8), dst * 256)
    assert torch.equal(out[dst], ops.fp8_dequant(q, s, torch.bfloat16))


@pytest.mark.parametrize("namespace", [b"", b"sixteen-byte-ns!", b"odd-namespace"])
def test_prefix_hash_bit_identical_to_hashlib(namespace):
    rng = np.random.default_rng(0)
    reqs = [rng.integers(0, 150_000, size=n).tolist() for n in (0, 63, 64, 300, 1024, 4096 + 17)]
    got = ops.prefix_hash(reqs, 64, namespace=namespace)
    for r, g in zip(reqs, got):
        assert g == chunk_keys_for_tokens(r, 64, namespace=namespace)


def fmix64(k):
    k ^= k >> np.uint64(33)
    k *= np.uint64(0xff51afd7ed558ccd)
    k ^= k >> np.uint64(33)
    k *= np.uint64(0xc4ceb9fe1a85ec53)
    k ^= k >> np.uint64(33)
    return k


def test_kv_checksum_matches_numpy_reference():
    pool = torch.randn(2, 2, 16, 16, 2, 64, dtype=torch.bfloat16, device="cuda")
    blocks = torch.tensor([3, 7, 11], device="cuda")
    got = ops.kv_checksum(pool, blocks).cpu().numpy().view(np.uint64)
    host = pool.cpu()
    with np.errstate(over="ignore"):
        for bi, b in enumerate(blocks.tolist()):
            for l in range(2):
                for p in range(2):
                    w = host[l, p, b].contiguous().view(torch.int64).numpy().view(np.uint64).reshape(-1)
                    idx = np.arange(w.size, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
                    ref = np.sum(fmix64(w ^ idx), dtype=np.uint64)
                    assert got[bi, l, p] == ref
    pool[0, 1, 7, 0, 0, 0] += 1
    assert ops.kv_checksum(pool, blocks)[1, 0, 1].item() != int(got[1, 0, 1].astype(np.int64))


def test_checksum_segment_parallel_path_equals_per_item_path():
    # 33,280-byte pages: two full 16 KiB segments and a partial one
    from tutti_b200._native import ops as _ops

    pool = torch.randn(3, 2, 10, 16, 8, 130, dtype=torch.bfloat16, device="cuda")
    blocks = torch.tensor([0, 4, 9], device="cuda")
    fast = ops.kv_checksum(pool, blocks)
    ptrs = ops._block_ptrs(pool, blocks, torch.arange(3))
    items = ops._items(ptrs, torch.zeros_like(ptrs), pool[0, 0, 0].numel() * 2)
    slow = _ops().checksum(items, 0).reshape(ptrs.shape)
    assert torch.equal(fast, slow)
