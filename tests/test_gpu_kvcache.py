"""Paged compressed KV cache: online page append (zs_kv_append_pages) is
byte-identical to the matrix encoder on each page, the pools decode back to
the appended K/V, and paged decode attention (zs_decode_attention_paged, with
dense tail pages) matches fp32 attention while sequences grow token by token."""
import math

import pytest
import torch

from zipserv_asplos26_b200.kvcache import BlockAllocator, PagedZipKVCache

TOL = 1e-3  # rel-L2 against the bf16-rounded fp32 reference


def test_block_allocator():
    a = BlockAllocator(4)
    got = [a.alloc() for _ in range(4)]
    assert sorted(got) == [0, 1, 2, 3] and a.num_free == 0
    with pytest.raises(RuntimeError):
        a.alloc()
    a.free(got[:2])
    assert a.num_free == 2
    with pytest.raises(ValueError):
        a.free([7])


def _kv(gen, T, Hkv, D=128):
    scale = torch.exp(torch.empty(Hkv, D, device="cuda").uniform_(math.log(0.1), math.log(4.0), generator=gen))
    return (torch.randn(T, Hkv, D, device="cuda", generator=gen) * scale).to(torch.bfloat16)


def _ref_attention(q, ks, vs, scale):
    outs = []
    for b, (k, v) in enumerate(zip(ks, vs)):
        Hq, Hkv = q.shape[1], k.shape[1]
        G = Hq // Hkv
        qf = q[b].float().view(Hkv, G, -1)
        s = torch.einsum("hgd,thd->hgt", qf, k.float()) * scale
        o = torch.einsum("hgt,thd->hgd", s.softmax(-1), v.float())
        outs.append(o.reshape(Hq, -1))
    return torch.stack(outs).to(torch.bfloat16).float()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.gpu
def test_page_append_matches_matrix_encoder(oracle):
    import numpy as np

    import zipserv_asplos26_b200 as zs
    gen = torch.Generator(device="cuda").manual_seed(11)
    Hkv = 2
    k, v = _kv(gen, 128, Hkv), _kv(gen, 128, Hkv)
    win = PagedZipKVCache.window_from(k)
    cache = PagedZipKVCache(num_blocks=4, max_batch=1, max_blocks_per_seq=4, num_kv_heads=Hkv, k_window=win,
                            v_window=PagedZipKVCache.window_from(v))
    cache.prefill(0, k, v)
    torch.cuda.synchronize()
    assert cache.check_errors() == 0
    pool = cache.k
    offs = pool.page_off.view(-1, 6).cpu()
    for j, blk in enumerate(cache.blocks[0]):
        for h in range(Hkv):
            P = blk * Hkv + h
            page = k[64 * j:64 * (j + 1), h].contiguous()          # [64 tokens, 128 dims]
            c = zs.compress(page, top=win)
            o = offs[P].tolist()
            assert o[2] - o[0] == c.tile_offsets_global[2].item() and o[4] - o[0] == c.total_hf
            assert o[5] - o[1] == c.total_full
            assert torch.equal(pool.sm[o[0]:o[4]], c.sign_mantissa[:c.total_hf])
            assert torch.equal(pool.full[o[1]:o[5]].view(torch.int16), c.compressed_full[:c.total_full].view(torch.int16))
            for bi in range(3):
                assert torch.equal(pool.b[bi][P * 128:(P + 1) * 128], getattr(c, f"bitmap{bi + 1}"))
            assert torch.equal(pool.mt_off[P * 16:(P + 1) * 16], c.tile_offsets_median)
            # and the CPU oracle's encoding of the same page with the same window
            e = oracle.encode(page.cpu().view(torch.int16).numpy().view(np.uint16), win.cpu().numpy())
            assert np.array_equal(pool.sm[o[0]:o[4]].cpu().numpy(), e.sign_mantissa)
            assert np.array_equal(pool.full[o[1]:o[5]].cpu().view(torch.int16).numpy().view(np.uint16), e.full)
            assert np.array_equal(pool.b[0][P * 128:(P + 1) * 128].view(torch.int64).cpu().numpy().view(np.uint64), e.bitmap1)


@pytest.mark.gpu
def test_paged_attention_while_sequences_grow():
    gen = torch.Generator(device="cuda").manual_seed(12)
    Hkv, Hq, D = 8, 32, 128
    prompts = [100, 64, 1]
    ks = [_kv(gen, T, Hkv) for T in prompts]
    vs = [_kv(gen, T, Hkv) for T in prompts]
    cache = PagedZipKVCache(num_blocks=16, max_batch=3, max_blocks_per_seq=4, num_kv_heads=Hkv,
                            k_window=PagedZipKVCache.window_from(ks[0]), v_window=PagedZipKVCache.window_from(vs[0]))
    for b in range(3):
        cache.prefill(b, ks[b], vs[b])
    scale = 1.0 / math.sqrt(D)
    checked = 0
    for step in range(72):
        if step in (0, 1, 27, 28, 63, 64, 71):
            q = torch.randn(3, Hq, D, device="cuda", generator=gen).to(torch.bfloat16)
            for splits in (0, 1):
                out = cache.attention(q, num_splits=splits)
                ref = _ref_attention(q, ks, vs, scale)
                assert _rel(out, ref) <= TOL, (step, splits, _rel(out, ref))
            checked += 1
        kn = torch.stack([_kv(gen, 1, Hkv)[0] for _ in range(3)])
        vn = torch.stack([_kv(gen, 1, Hkv)[0] for _ in range(3)])
        cache.append(kn, vn)
        for b in range(3):
            ks[b] = torch.cat([ks[b], kn[b:b + 1]])
            vs[b] = torch.cat([vs[b], vn[b:b + 1]])
    torch.cuda.synchronize()
    assert cache.check_errors() == 0
    assert checked == 7
    for b in range(3):
        k, v = cache.dense(b)
        assert torch.equal(k.view(torch.int16), ks[b].view(torch.int16))
        assert torch.equal(v.view(torch.int16), vs[b].view(torch.int16))
    # freeing a sequence returns its blocks
    n0 = cache.alloc.num_free
    cache.free(2)
    assert cache.alloc.num_free == n0 + (prompts[2] + 72) // 64


@pytest.mark.gpu
def test_pool_overflow_sets_error_bit():
    gen = torch.Generator(device="cuda").manual_seed(13)
    k, v = _kv(gen, 256, 1), _kv(gen, 256, 1)
    cache = PagedZipKVCache(num_blocks=4, max_batch=1, max_blocks_per_seq=4, num_kv_heads=1,
                            k_window=PagedZipKVCache.window_from(k), v_window=PagedZipKVCache.window_from(v),
                            hf_bytes_per_page=2048, full_elems_per_page=64)
    cache.prefill(0, k, v)
    torch.cuda.synchronize()
    assert cache.check_errors() & 2


PAGED_LONG = [(32, 4129), (8, 16417), (1, 32801)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,T", PAGED_LONG, ids=[f"B{b}-T{t}" for b, t in PAGED_LONG])
def test_paged_attention_long_contexts(B, T):
    """The bench's paged cases (config-5 shapes, lengths T % 64 == 33 so each
    sequence ends in a dense tail page) against attention on the original K/V."""
    gen = torch.Generator(device="cuda").manual_seed(100 + B)
    Hq, Hkv, D = 32, 8, 128
    ks = [_kv(gen, T, Hkv) for _ in range(B)]
    vs = [_kv(gen, T, Hkv) for _ in range(B)]
    blocks = (T + 63) // 64
    cache = PagedZipKVCache(num_blocks=B * blocks, max_batch=B, max_blocks_per_seq=blocks, num_kv_heads=Hkv,
                            k_window=PagedZipKVCache.window_from(ks[0]), v_window=PagedZipKVCache.window_from(vs[0]),
                            full_elems_per_page=2048, device=torch.device("cuda"))
    for b in range(B):
        cache.prefill(b, ks[b], vs[b])
    q = torch.randn(B, Hq, D, device="cuda", generator=gen).to(torch.bfloat16)
    ref = _ref_attention(q, ks, vs, 1.0 / math.sqrt(D))
    for splits in (1, 0):
        out = cache.attention(q, num_splits=splits)
        torch.cuda.synchronize()
        assert _rel(out, ref) <= TOL, (splits, _rel(out, ref))
