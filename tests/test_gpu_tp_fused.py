"""Row-parallel ZipGEMM with the all-reduce fused into the kernel
(zs_zipgemm_allreduce), one process per GPU, world sizes 2..device count,
with both exchange schemes (all-to-all, and reduce-scatter + all-gather by
tile owner).

The expected output is exact: every rank's partial is its own ZipGEMM of its
K shard (zs_zipgemm, bf16), and the fused kernel must return, on every rank,
bf16(sum in rank order of the bf16 partials, in fp32). The checks cover
consecutive calls with different activations (the exchange buffer halves
alternate), a CUDA graph of several calls replayed twice, a 70B O-projection
shape, and the layer wrapper (RowParallelZipLinear(fused=True)).

Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expected(partial, world):
    parts = [torch.empty_like(partial) for _ in range(world)]
    dist.all_gather(parts, partial)
    acc = parts[0].float()
    for p in parts[1:]:
        acc = acc + p.float()
    return acc.to(torch.bfloat16)


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        import zipserv_asplos26_b200 as zs
        from zipserv_asplos26_b200.tp import AllReduceBuffers, RowParallelZipLinear, shard_cols, zipgemm_allreduce

        out = {}
        for (M, K, N) in [(4096, 4096, 128), (8192, 8192, 16), (1024, 2048, 7)]:
            g = torch.Generator().manual_seed(7)
            w = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16)
            k = K // world
            c = zs.compress(shard_cols(w, rank, world).to(dev))
            bufs = AllReduceBuffers(M, N, device=dev)
            worst = 0
            for call in range(3):
                xg = torch.Generator().manual_seed(100 + call)
                x = torch.randn(N, K, generator=xg).to(torch.bfloat16)[:, rank * k:(rank + 1) * k].contiguous().to(dev)
                y = zipgemm_allreduce(c, x, bufs)
                ref = _expected(zs.zipgemm(c, x), world)
                torch.cuda.synchronize()
                worst = max(worst, int((y != ref).sum()))
            # a graph of four calls on two activations, replayed twice
            xs = []
            for i in range(2):
                xg = torch.Generator().manual_seed(200 + i)
                xs.append(torch.randn(N, K, generator=xg).to(torch.bfloat16)[:, rank * k:(rank + 1) * k]
                          .contiguous().to(dev))
            ys = [torch.empty(N, M, dtype=torch.bfloat16, device=dev) for _ in range(4)]
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    for i in range(4):
                        zipgemm_allreduce(c, xs[i % 2], bufs, out=ys[i])
                graph.replay()
                graph.replay()
                s.synchronize()
            for i in range(4):
                ref = _expected(zs.zipgemm(c, xs[i % 2]), world)
                torch.cuda.synchronize()
                worst = max(worst, int((ys[i] != ref).sum()))
            out[(M, K, N)] = worst
            dist.barrier()
            del graph
            bufs.close()

        # the layer wrapper, against the unfused layer (ZipGEMM + NCCL all-reduce)
        g = torch.Generator().manual_seed(9)
        w = (torch.randn(2048, 4096, generator=g) * 0.02).to(torch.bfloat16)
        shard = shard_cols(w, rank, world).to(dev)
        fused = RowParallelZipLinear(shard, fused=True)
        x = torch.randn(32, 4096 // world, generator=g).to(torch.bfloat16).to(dev)
        y = fused(x)
        parts = zs.zipgemm(fused.weight, x)
        out["layer"] = int((y != _expected(parts, world)).sum())
        torch.cuda.synchronize()
        dist.barrier()
        for b in fused._bufs.values():
            b.close()
        q.put((rank, out))
        dist.barrier()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world,scheme", [(2, None), (2, "owner"), (4, None), (4, "all2all"), (8, None)])
def test_gpu_zipgemm_allreduce_matches_partials(world, scheme, monkeypatch):
    """scheme None: the default exchange for the world size (all-to-all at 2
    ranks, reduce-scatter + all-gather by tile owner from 3 on); "owner" /
    "all2all" force the other one through ZS_ALLREDUCE_SCHEME."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if scheme:
        monkeypatch.setenv("ZS_ALLREDUCE_SCHEME", scheme)
    else:
        monkeypatch.delenv("ZS_ALLREDUCE_SCHEME", raising=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, out in res:
        assert isinstance(out, dict), (rank, out)
        assert all(v == 0 for v in out.values()), (rank, out)
