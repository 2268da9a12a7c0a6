"""Tensor-parallel sharding + all-reduce logic on CPU ranks (gloo, world sizes 2, 4, 8).

The GEMM backend is injected (dense fp32 matmul on the decompressed shard is
replaced by a plain matmul of the dense shard), so these tests check the
sharding and the reduction, not the kernels (those are covered on the GPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dense_gemm(w, x, out=None):
    y = x.float() @ w.float().t()
    if out is not None:
        out.copy_(y)
        return out
    return y


def _identity(w):
    return w


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from zipserv_asplos26_b200.tp import (ColumnParallelZipLinear, RowParallelZipLinear, shard_cols,
                                              shard_rows)
        torch.manual_seed(0)
        M, K, N = 512, 1024, 5
        w = torch.randn(M, K)
        x = torch.randn(N, K)
        ref = x @ w.t()
        col = ColumnParallelZipLinear(shard_rows(w, rank, world), gemm=_dense_gemm, compressor=_identity)
        y_col = col(x)
        gathered = [torch.empty_like(y_col) for _ in range(world)]
        dist.all_gather(gathered, y_col)
        err_col = float((torch.cat(gathered, dim=1) - ref).abs().max())
        row = RowParallelZipLinear(shard_cols(w, rank, world), gemm=_dense_gemm, compressor=_identity)
        k = K // world
        y_row = row(x[:, rank * k:(rank + 1) * k].contiguous())
        err_row = float((y_row - ref).abs().max())
        q.put((rank, err_col, err_row))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), None))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_column_and_row_parallel_match_dense(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ec, er in res:
        assert isinstance(ec, float), ec
        assert ec < 1e-4 and er < 1e-4, (rank, ec, er)


def test_shard_validation():
    from zipserv_asplos26_b200.tp import shard_cols, shard_rows
    w = torch.zeros(192, 256)
    assert shard_rows(w, 1, 3).shape == (64, 256)
    assert shard_cols(w, 3, 4).shape == (192, 64)
    with pytest.raises(ValueError):
        shard_rows(w, 0, 2)       # 96 rows per rank
    with pytest.raises(ValueError):
        shard_cols(w, 0, 3)


def test_tp_layer_shapes_single_rank():
    from zipserv_asplos26_b200.tp import LLAMA8B_SHAPES, TPLayerGemms
    small = {k: (m // 16, kk // 16) for k, (m, kk) in LLAMA8B_SHAPES.items()}
    small = {k: ((m + 63) // 64 * 64, (kk + 63) // 64 * 64) for k, (m, kk) in small.items()}
    lay = TPLayerGemms(small, gemm=_dense_gemm, compressor=_identity, dtype=torch.float32)
    xs = {n: torch.randn(*s) for n, s in lay.input_shapes(3).items()}
    ys = lay.run(xs)
    for n, y in ys.items():
        assert y.shape == (3, small[n][0])


def _ref_attention(q, k, v, seqlens, num_kv_heads):
    """fp32 decode attention: q [B, Hq, D], k/v [B, T, Hkv, D] (dense, uncompressed)."""
    B, Hq, D = q.shape
    G = Hq // num_kv_heads
    out = torch.empty(B, Hq, D)
    for b in range(B):
        t = int(seqlens[b])
        for h in range(Hq):
            kk, vv = k[b, :t, h // G].float(), v[b, :t, h // G].float()
            p = torch.softmax(kk @ q[b, h].float() / D ** 0.5, 0)
            out[b, h] = p @ vv
    return out


def _attn_worker(rank, world, port, q_out, batch_shards=1):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from zipserv_asplos26_b200.tp import KVHeadParallelDecodeAttention
        torch.manual_seed(1)
        B, T, Hq, Hkv, D = 4, 40, 16, 8, 16
        q = torch.randn(B, Hq, D)
        k, v = torch.randn(B, T, Hkv, D), torch.randn(B, T, Hkv, D)
        seq = torch.tensor([40, 17, 1, 33])
        ref = _ref_attention(q, k, v, seq, Hkv)
        att = KVHeadParallelDecodeAttention(Hq, Hkv, compress_kv=_identity, attention=_ref_attention,
                                            batch_shards=batch_shards)
        att.load_kv(att.shard_kv(k), att.shard_kv(v))
        o = att.gather_batch(att(att.shard_q(q), seq))     # this rank's heads, every sequence
        gathered = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(gathered, o)
        hs = att.head_shards
        full = torch.cat(gathered[:hs], dim=1)             # the head groups of batch shard 0 cover all heads
        q_out.put((rank, float((full - ref).abs().max()), att.q_heads, att.batch_range(B)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q_out.put((rank, repr(e), None, None))


ATTN_GRIDS = [(2, 1), (4, 1), (8, 1), (4, 2), (8, 4), (8, 2)]


@pytest.mark.parametrize("world,batch_shards", ATTN_GRIDS, ids=[f"w{w}-b{b}" for w, b in ATTN_GRIDS])
def test_kv_head_and_batch_parallel_attention_matches_full(world, batch_shards):
    """Sharding decode attention by KV head (with its query-head group) and by
    batch, then reassembling the ranks' outputs, reproduces full attention
    (gloo ranks on CPU; the per-shard kernel runs in the GPU tests)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_attn_worker, args=(r, world, port, q, batch_shards)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    hs = world // batch_shards
    G, per = 2, 8 // hs
    for rank, err, heads, brange in res:
        assert not isinstance(err, str), err
        assert err < 1e-5
        h = rank % hs
        assert heads == (h * per * G, (h + 1) * per * G)
        nb = 4 // batch_shards
        assert brange == ((rank // hs) * nb, (rank // hs + 1) * nb)
