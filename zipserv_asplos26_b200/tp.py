"""Tensor-parallel ZipGEMM layers (new relative to the reference, which has no
collectives): column-parallel projections (QKV, gate_up) split W by output rows
and need no communication; row-parallel projections (O, down) split W by K and
sum the per-rank partial outputs with one all-reduce (NCCL over NVLink on GPUs;
any torch.distributed backend works, gloo is used by the CPU tests).

Each rank compresses only its own shard (its own exponent window), exactly as a
per-rank checkpoint would be compressed."""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def _rank_world(group=None):
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def shard_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [M/world * rank, M/world * (rank+1)) of W (column-parallel shard)."""
    M = w.shape[0]
    if M % world or (M // world) % 64:
        raise ValueError(f"M={M} must split into multiples of 64 over {world} ranks")
    m = M // world
    return w[rank * m:(rank + 1) * m].contiguous()


def shard_cols(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns [K/world * rank, ...) of W (row-parallel shard)."""
    K = w.shape[1]
    if K % world or (K // world) % 64:
        raise ValueError(f"K={K} must split into multiples of 64 over {world} ranks")
    k = K // world
    return w[:, rank * k:(rank + 1) * k].contiguous()


class AllReduceBuffers:
    """Exchange buffers of the fused row-parallel all-reduce (zs_zipgemm_allreduce)
    for outputs of M x N: one buffer per rank in its own GPU memory, mapped
    into every other rank through CUDA IPC (the handles travel over the
    process group), plus this rank's per-tile exchange counters. Creating one
    is collective over `group`; make it before any CUDA-graph capture."""

    def __init__(self, M: int, N: int, group=None, device=None):
        import ctypes as C
        from ._lib import check, lib
        self.rank, self.world = _rank_world(group)
        if self.world < 2:
            raise ValueError("the fused all-reduce needs at least 2 ranks")
        L = lib()
        self.M, self.N = M, N
        nbytes = L.zs_zipgemm_allreduce_buffer_bytes(M, N, self.world)
        if nbytes == 0:
            raise ValueError(f"no exchange buffer for M={M} N={N} world={self.world}")
        handle = C.create_string_buffer(L.zs_peer_handle_bytes())
        own = C.c_void_p()
        check(L.zs_peer_alloc(nbytes, C.byref(own), handle), "zs_peer_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._own = own.value
        self._opened = []
        ptrs = []
        for j, h in enumerate(handles):
            if j == self.rank:
                ptrs.append(self._own)
                continue
            p = C.c_void_p()
            check(L.zs_peer_open(C.create_string_buffer(h, len(h)), C.byref(p)), "zs_peer_open")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.peer_array = (C.c_void_p * self.world)(*ptrs)
        self.epoch = torch.zeros(L.zs_zipgemm_allreduce_counters(M, N), dtype=torch.int32, device=device)

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every rank's last call)."""
        from ._lib import lib
        L = lib()
        for p in self._opened:
            L.zs_peer_close(p)
        self._opened = []
        if self._own:
            L.zs_peer_free(self._own)
            self._own = None


def zipgemm_allreduce(c, x: torch.Tensor, bufs: AllReduceBuffers, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y[N, M] = sum over ranks of x_r @ W_r^T, the all-reduce fused into the
    ZipGEMM (zs_zipgemm_allreduce): `c` is this rank's compressed K shard of W,
    `x` its [N, K_shard] slice of the activations. Every rank gets the same y."""
    from ._lib import check, lib
    from .codec import _check_2d_bf16
    _check_2d_bf16(x, "x")
    N, K = x.shape
    if K != c.cols or (c.rows, N) != (bufs.M, bufs.N):
        raise ValueError("x / W shard / exchange buffers disagree on M, N or K")
    if out is None:
        out = torch.empty(N, c.rows, dtype=torch.bfloat16, device=x.device)
    _check_2d_bf16(out, "out")
    check(lib().zs_zipgemm_allreduce(torch.cuda.current_stream().cuda_stream, c.sign_mantissa.data_ptr(),
                                     c.compressed_full.data_ptr(), c.bitmap1.data_ptr(), c.bitmap2.data_ptr(),
                                     c.bitmap3.data_ptr(), c.tile_offsets_median.data_ptr(),
                                     c.tile_offsets_global.data_ptr(), c.max_high_freq_count, c.max_full_count,
                                     c.start_exp, x.data_ptr(), out.data_ptr(), c.rows, N, K, bufs.world, bufs.rank,
                                     bufs.peer_array, bufs.epoch.data_ptr(), None), "zs_zipgemm_allreduce")
    return out


def _zipgemm_backend(c, x, out=None):
    from .codec import zipgemm
    return zipgemm(c, x, out=out)


def _compress_backend(w):
    from .codec import compress
    return compress(w)


class ColumnParallelZipLinear:
    """y_local[N, M/world] = x[N, K] @ W_shard^T; no collective."""

    def __init__(self, w_shard: torch.Tensor, gemm: Callable = _zipgemm_backend,
                 compressor: Callable = _compress_backend, group=None):
        self.gemm = gemm
        self.group = group
        self.weight = compressor(w_shard)
        self.out_features = w_shard.shape[0]
        self.in_features = w_shard.shape[1]

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.gemm(self.weight, x, out=out)


class RowParallelZipLinear:
    """y[N, M] = sum over ranks of x_local[N, K/world] @ W_shard^T (all-reduce).

    fused=True (CUDA ranks): one zs_zipgemm_allreduce per call, the exchange
    over NVLink inside the ZipGEMM; the exchange buffers for each token count
    N are made on the first call with that N (collective: every rank calls
    with the same N). fused=False: ZipGEMM, then torch.distributed.all_reduce
    (any backend; the CPU tests use gloo)."""

    def __init__(self, w_shard: torch.Tensor, gemm: Callable = _zipgemm_backend,
                 compressor: Callable = _compress_backend, group=None, fused: bool = False):
        self.gemm = gemm
        self.group = group
        self.fused = fused
        self.weight = compressor(w_shard)
        self.out_features = w_shard.shape[0]
        self.in_features = w_shard.shape[1]
        self._bufs = {}

    def __call__(self, x_local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        _, world = _rank_world(self.group)
        if self.fused and world > 1:
            N = x_local.shape[0]
            if N not in self._bufs:
                self._bufs[N] = AllReduceBuffers(self.out_features, N, group=self.group, device=x_local.device)
            return zipgemm_allreduce(self.weight, x_local, self._bufs[N], out=out)
        y = self.gemm(self.weight, x_local, out=out)
        if world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y


# Llama-3.1-70B projection shapes: (out_features, in_features)
LLAMA70B_SHAPES = {"qkv": (10240, 8192), "o": (8192, 8192), "gate_up": (57344, 8192), "down": (8192, 28672)}
LLAMA8B_SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


class TPLayerGemms:
    """The four weight GEMMs of one decoder layer, tensor-parallel:
    QKV and gate_up column-parallel, O and down row-parallel (+ all-reduce,
    fused into the ZipGEMM when fused=True).
    Weights are generated per rank from a seed (synthetic, N(0, sigma))."""

    def __init__(self, shapes=LLAMA70B_SHAPES, seed: int = 0, sigma: float = 0.02, device=None,
                 gemm: Callable = _zipgemm_backend, compressor: Callable = _compress_backend,
                 dtype=torch.bfloat16, group=None, fused: bool = False):
        rank, world = _rank_world(group)
        self.rank, self.world = rank, world
        self.layers = {}
        for i, (name, (M, K)) in enumerate(shapes.items()):
            col = name in ("qkv", "gate_up")
            m = M // world if col else M
            k = K if col else K // world
            if (m % 64) or (k % 64):
                raise ValueError(f"{name}: shard {m}x{k} is not a multiple of 64")
            g = torch.Generator(device=device if device is not None else "cpu")
            g.manual_seed(seed * 1000 + i * 16 + rank)
            w = (torch.randn(m, k, generator=g, device=device) * sigma).to(dtype)
            if col:
                self.layers[name] = ColumnParallelZipLinear(w, gemm=gemm, compressor=compressor, group=group)
            else:
                self.layers[name] = RowParallelZipLinear(w, gemm=gemm, compressor=compressor, group=group,
                                                         fused=fused)

    def input_shapes(self, n_tokens: int):
        """Activation shapes each projection consumes on this rank."""
        return {name: (n_tokens, lay.in_features) for name, lay in self.layers.items()}

    def run(self, xs: dict):
        return {name: self.layers[name](xs[name]) for name in self.layers}


def _compress_kv_backend(x):
    from .attention import compress_kv
    return compress_kv(x)


def _decode_attention_backend(q, k, v, seqlens, num_kv_heads):
    from .attention import decode_attention
    return decode_attention(q, k, v, seqlens, num_kv_heads)


class KVHeadParallelDecodeAttention:
    """Decode attention sharded by KV head and by batch (no collective in the
    attention itself). The ranks form a grid of batch_shards x head_shards
    (head_shards = world / batch_shards): rank r owns KV heads
    [h Hkv/hs, (h+1) Hkv/hs) with h = r % hs, together with the G = Hq/Hkv query
    heads of each, for the sequences [b B/bs, (b+1) B/bs) with b = r // hs. With
    batch_shards = 1 a rank's output heads are contiguous for the whole batch and
    feed the row-parallel O projection directly; batch sharding serves more
    ranks than KV heads (or balances uneven sequence lengths), and
    gather_batch() reassembles a head group's outputs over the batch. Each rank
    compresses its own K/V slice (its own exponent window), as a per-rank cache
    would be."""

    def __init__(self, num_heads: int, num_kv_heads: int, group=None,
                 compress_kv: Callable = _compress_kv_backend, attention: Callable = _decode_attention_backend,
                 batch_shards: int = 1, rank: Optional[int] = None, world: Optional[int] = None):
        # rank / world default to the process group's; given explicitly, one
        # process can stand in for any rank of a grid (tests, offline sharding)
        grank, gworld = _rank_world(group)
        rank = grank if rank is None else rank
        world = gworld if world is None else world
        if batch_shards < 1 or world % batch_shards:
            raise ValueError(f"{batch_shards} batch shards do not divide {world} ranks")
        hs = world // batch_shards
        if num_heads % num_kv_heads or num_kv_heads % hs:
            raise ValueError(f"{num_kv_heads} KV heads do not split over {hs} head shards "
                             f"(or {num_heads} heads are not a multiple of them)")
        self.group, self.world = group, world
        self.batch_shards, self.head_shards = batch_shards, hs
        self.bshard, self.hshard = rank // hs, rank % hs
        self.G = num_heads // num_kv_heads
        self.kv_local = num_kv_heads // hs
        self.kv0 = self.hshard * self.kv_local
        self.compress_kv, self.attention = compress_kv, attention
        self.k = self.v = None

    def batch_range(self, batch: int):
        """Sequences [start, stop) this rank serves out of `batch`."""
        if batch % self.batch_shards:
            raise ValueError(f"batch {batch} does not split into {self.batch_shards} shards")
        n = batch // self.batch_shards
        return self.bshard * n, (self.bshard + 1) * n

    def shard_batch(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's sequences of a batch-leading tensor (q, K/V or seqlens)."""
        a, b = self.batch_range(x.shape[0])
        return x[a:b].contiguous()

    def gather_batch(self, out_local: torch.Tensor) -> torch.Tensor:
        """All sequences of this rank's heads: all-gather over the ranks that
        hold the same heads for the other batch shards (collective; identity
        without batch sharding)."""
        if self.batch_shards == 1:
            return out_local
        parts = [torch.empty_like(out_local) for _ in range(self.world)]
        dist.all_gather(parts, out_local.contiguous(), group=self.group)
        return torch.cat([parts[b * self.head_shards + self.hshard] for b in range(self.batch_shards)], dim=0)

    @property
    def q_heads(self):
        """Query-head range [start, stop) this rank computes."""
        return self.kv0 * self.G, (self.kv0 + self.kv_local) * self.G

    def shard_kv(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's sequences and KV heads of a [B, T, Hkv, D] tensor."""
        a, b = self.batch_range(x.shape[0])
        return x[a:b, :, self.kv0:self.kv0 + self.kv_local].contiguous()

    def shard_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's sequences and query heads of a [B, Hq, D] tensor."""
        a, b = self.q_heads
        s0, s1 = self.batch_range(q.shape[0])
        return q[s0:s1, a:b].contiguous()

    def load_kv(self, k_local: torch.Tensor, v_local: torch.Tensor):
        """Compress this rank's K and V ([B, T, Hkv/world, D])."""
        self.k, self.v = self.compress_kv(k_local), self.compress_kv(v_local)

    def __call__(self, q_local: torch.Tensor, seqlens: torch.Tensor) -> torch.Tensor:
        """q_local from shard_q; seqlens of the whole batch or of this rank's
        sequences. Returns [B / batch_shards, Hq / head_shards, D]."""
        if self.k is None:
            raise RuntimeError("load_kv first")
        if seqlens.shape[0] != q_local.shape[0]:
            seqlens = self.shard_batch(seqlens)
        return self.attention(q_local, self.k, self.v, seqlens, self.kv_local)
