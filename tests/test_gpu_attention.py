"""Compressed-KV decode attention vs an fp32 torch reference on the original K/V.

Decode is lossless, so the reference is exact attention on the uncompressed
cache, rounded to bf16 like any bf16-output kernel."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-3  # rel-L2 against the bf16-rounded fp32 reference


def make_kv(B, T, Hkv, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.empty(D, device="cuda").uniform_(math.log(0.1), math.log(4.0), generator=g))
    return (torch.randn(B, T, Hkv, D, generator=g, device="cuda") * s).to(torch.bfloat16)


def reference(q, k, v, lens, scale):
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    out = torch.empty(B, Hq, D, dtype=torch.float64, device=q.device)
    for b in range(B):
        L = int(lens[b])
        kk = k[b, :L].double().permute(1, 0, 2)  # Hkv, L, D
        vv = v[b, :L].double().permute(1, 0, 2)
        qq = q[b].double().view(Hkv, G, D)
        s = torch.einsum("hgd,htd->hgt", qq, kk) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgt,htd->hgd", p, vv).reshape(Hq, D)
    return out


def rel_l2(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


@pytest.mark.parametrize("B,T,splits", [(1, 64, 1), (2, 100, 1), (2, 1000, 0), (3, 1500, 4), (1, 4096, 0),
                                        (8, 333, 0), (2, 1, 0)])
def test_decode_attention_matches_fp32_reference(B, T, splits):
    import zipserv_asplos26_b200 as zs
    Hq, Hkv, D = 32, 8, 128
    k = make_kv(B, T, Hkv, D, seed=T)
    v = make_kv(B, T, Hkv, D, seed=T + 1)
    q = torch.randn(B, Hq, D, device="cuda").to(torch.bfloat16)
    kc = zs.compress_kv(k)
    vc = zs.compress_kv(v)
    lens = torch.full((B,), T, dtype=torch.int32, device="cuda")
    if B > 1:
        lens[0] = max(1, T // 2)   # ragged batch
    out = zs.decode_attention(q, kc, vc, lens, Hkv, num_splits=splits)
    torch.cuda.synchronize()
    ref = reference(q, k, v, lens.cpu(), 1.0 / math.sqrt(D)).to(torch.bfloat16)
    assert rel_l2(out, ref) <= TOL


def test_flash_attn_with_kvcache_descriptor_api():
    import zipserv_asplos26_b200 as zs
    B, T, Hq, Hkv, D = 2, 256, 32, 8, 128
    k = make_kv(B, T, Hkv, D, 5)
    v = make_kv(B, T, Hkv, D, 6)
    q = torch.randn(B, 1, Hq, D, device="cuda").to(torch.bfloat16)
    kc, vc = zs.compress_kv(k), zs.compress_kv(v)
    out = zs.flash_attn_with_kvcache(q, cache_seqlens=T, zipserv_k=kc.descriptor(), zipserv_v=vc.descriptor(),
                                     zipserv_num_heads_k=Hkv)
    ref = reference(q.view(B, Hq, D), k, v, [T] * B, 1.0 / math.sqrt(D)).to(torch.bfloat16)
    assert out.shape == q.shape
    assert rel_l2(out.view(B, Hq, D), ref) <= TOL


def test_decode_attention_kv_round_trip_is_lossless():
    import zipserv_asplos26_b200 as zs
    k = make_kv(2, 200, 8, 128, 9)
    flat, _, _ = zs.pad_kv_by_kv_head(k)
    kc = zs.compress_kv(k)
    assert torch.equal(zs.decompress(kc).view(torch.int16), flat.view(torch.int16))


def test_kv_head_parallel_attention_single_rank_uses_the_kernel():
    """KVHeadParallelDecodeAttention with its default backends (compress_kv +
    decode_attention): one rank owns every head and matches the fp32 reference."""
    from zipserv_asplos26_b200.tp import KVHeadParallelDecodeAttention
    B, T, Hq, Hkv, D = 2, 300, 32, 8, 128
    k, v = make_kv(B, T, Hkv, D, 21), make_kv(B, T, Hkv, D, 22)
    q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(23)).to(
        torch.bfloat16)
    lens = torch.tensor([300, 129], dtype=torch.int32, device="cuda")
    att = KVHeadParallelDecodeAttention(Hq, Hkv)
    att.load_kv(att.shard_kv(k), att.shard_kv(v))
    out = att(att.shard_q(q), lens)
    ref = reference(q, k, v, lens, 1.0 / math.sqrt(D)).to(torch.bfloat16)
    assert rel_l2(out, ref) <= TOL


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 8), (64, 8), (6, 2)])
def test_decode_attention_query_group_sizes(Hq, Hkv):
    """Query groups G = Hq / Hkv of 1, 2, 8 and 3 (the MMA tiles hold up to 8
    query heads in their columns; unused columns must not leak into the output)."""
    import zipserv_asplos26_b200 as zs
    B, T, D = 2, 700, 128
    k = make_kv(B, T, Hkv, D, seed=31 + Hq)
    v = make_kv(B, T, Hkv, D, seed=32 + Hq)
    q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(Hq)).to(
        torch.bfloat16)
    lens = torch.tensor([700, 333], dtype=torch.int32, device="cuda")
    for splits in (1, 0):
        out = zs.decode_attention(q, zs.compress_kv(k), zs.compress_kv(v), lens, Hkv, num_splits=splits)
        ref = reference(q, k, v, lens.cpu(), 1.0 / math.sqrt(D)).to(torch.bfloat16)
        assert rel_l2(out, ref) <= TOL, (Hq, Hkv, splits)
