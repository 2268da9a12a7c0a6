"""Paged compressed KV cache with online page append.

The reference compresses a whole KV cache at once in its head-major layout
(kernel_benchmark/bench_zipserv_decode_attention.py:347-354) and its online
benchmark re-runs the matrix encoder pipeline per step
(kernel_benchmark/bench_kv_cache_zipserv_compress_token_scaling.cu:1606-1647).
Serving needs a cache that grows one token at a time, so here:

* K and V each live in a page pool (`zs_kv_append_pages` in the C ABI): a
  physical page is 64 tokens x 128 dims of one KV head, compressed with the
  pool's fixed exponent window, at slot `block * Hkv + head`; its streams are
  appended to shared stream pools.
* A sequence owns a list of blocks (one block = 64 tokens of every KV head),
  recorded in a block table as in paged attention.
* New tokens go to a dense tail page per sequence; when it holds 64 tokens it
  is compressed into a fresh block in one kernel launch for the whole batch.
* `attention()` runs the paged decode-attention kernel, which decodes the
  compressed pages and reads the dense tail page directly.

All host bookkeeping (lengths, block lists) is mirrored on the host so no call
synchronises the GPU.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import torch

from ._lib import check, lib
from .codec import analyze_exponents

D_HEAD = 128


class ZsKvPool(C.Structure):
    _fields_ = [("d_sm", C.c_void_p), ("d_full", C.c_void_p), ("d_b1", C.c_void_p), ("d_b2", C.c_void_p),
                ("d_b3", C.c_void_p), ("d_mt_off", C.c_void_p), ("d_page_off", C.c_void_p),
                ("d_cursor", C.c_void_p), ("hf_capacity", C.c_int64), ("full_capacity", C.c_int64),
                ("num_pages", C.c_int), ("start_exp", C.c_int), ("d_top7", C.c_void_p)]


_P = C.c_void_p
_SIGS = {
    "zs_kv_append_pages": ([_P, C.POINTER(ZsKvPool), _P, C.c_int, C.c_int, C.c_int, C.c_int, _P, _P], C.c_int),
    "zs_decode_attention_paged": ([_P, _P, C.POINTER(ZsKvPool), C.POINTER(ZsKvPool), _P, C.c_int, _P, _P, _P]
                                  + [C.c_int] * 5 + [C.c_float, C.c_int, _P, C.c_size_t, _P, _P, _P], C.c_int),
    "zs_decode_attention_workspace_bytes": ([C.c_int] * 4, C.c_size_t),
    "zs_decode_attention_default_splits": ([C.c_int] * 3, C.c_int),
}


def _fn(name):
    f = getattr(lib(), name)
    f.argtypes, f.restype = _SIGS[name]
    return f


def _stream():
    return torch.cuda.current_stream().cuda_stream


class BlockAllocator:
    """Free list of physical blocks (host only)."""

    def __init__(self, num_blocks: int):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, -1, -1))

    def alloc(self) -> int:
        if not self._free:
            raise RuntimeError("KV cache is out of blocks")
        return self._free.pop()

    def free(self, blocks: List[int]):
        for b in blocks:
            if not 0 <= b < self.num_blocks:
                raise ValueError(f"block {b} out of range")
        self._free.extend(reversed(blocks))

    @property
    def num_free(self) -> int:
        return len(self._free)


class _Pool:
    """Device arrays of one page pool (K or V)."""

    def __init__(self, num_pages: int, top: torch.Tensor, hf_bytes: int, full_elems: int, device):
        if hf_bytes >= 2 ** 31 or full_elems >= 2 ** 31:
            raise ValueError("stream pools are limited to 2**31 - 1 bytes / elements (int32 page offsets)")
        self.top = top.to(device=device, dtype=torch.int32).contiguous()
        top_host = self.top.cpu().tolist()
        self.start_exp = (int(top_host[0]) - 1) & 0xFF
        self.sm = torch.zeros(hf_bytes + 16, dtype=torch.uint8, device=device)
        self.full = torch.zeros(full_elems + 8, dtype=torch.bfloat16, device=device)
        self.b = [torch.zeros(num_pages * 2 * 64, dtype=torch.uint64, device=device) for _ in range(3)]
        self.mt_off = torch.zeros(num_pages * 2 * 8, dtype=torch.int32, device=device)
        self.page_off = torch.zeros(num_pages * 6, dtype=torch.int32, device=device)
        self.cursor = torch.zeros(4, dtype=torch.int64, device=device)   # next hf, next fallback, max hf, max fallback per GT
        self.st = ZsKvPool(self.sm.data_ptr(), self.full.data_ptr(), self.b[0].data_ptr(), self.b[1].data_ptr(),
                           self.b[2].data_ptr(), self.mt_off.data_ptr(), self.page_off.data_ptr(),
                           self.cursor.data_ptr(), hf_bytes, full_elems, num_pages, self.start_exp,
                           self.top.data_ptr())


class PagedZipKVCache:
    """Compressed K/V cache for up to `max_batch` sequences of up to
    `max_blocks_per_seq * 64` tokens, `num_kv_heads` heads of 128 dims.

    `k_window` / `v_window` are the pools' fixed 7-exponent windows (int32[7]);
    `window_from(sample)` picks one from a sample with the extension's rule,
    as the reference picks one window per K or V tensor. Pool sizes default to
    8 KB of sign/mantissa bytes and 1 K fallback elements per page (a page is
    16 KB dense); a page that does not fit sets an error bit (see
    `check_errors`)."""

    def __init__(self, num_blocks: int, max_batch: int, max_blocks_per_seq: int, num_kv_heads: int,
                 k_window: torch.Tensor, v_window: torch.Tensor, hf_bytes_per_page: int = 8192,
                 full_elems_per_page: int = 1024, device="cuda"):
        self.device = torch.device(device)
        self.Hkv = num_kv_heads
        self.max_batch = max_batch
        self.max_blocks = max_blocks_per_seq
        self.alloc = BlockAllocator(num_blocks)
        pages = num_blocks * num_kv_heads
        self.k = _Pool(pages, k_window, pages * hf_bytes_per_page, pages * full_elems_per_page, self.device)
        self.v = _Pool(pages, v_window, pages * hf_bytes_per_page, pages * full_elems_per_page, self.device)
        self.block_table = torch.zeros(max_batch, max_blocks_per_seq, dtype=torch.int32, device=self.device)
        self.seqlens = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
        self.tail_k = torch.zeros(max_batch, 64, num_kv_heads, D_HEAD, dtype=torch.bfloat16, device=self.device)
        self.tail_v = torch.zeros_like(self.tail_k)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.lengths = [0] * max_batch
        self.blocks: List[List[int]] = [[] for _ in range(max_batch)]

    @staticmethod
    def window_from(sample: torch.Tensor) -> torch.Tensor:
        """7-exponent window of a bf16 CUDA sample (the extension's rule)."""
        return analyze_exponents(sample.reshape(-1, D_HEAD).contiguous(), rule="ext")

    # ---------------------------------------------------------------- writes
    def _append(self, x_k: torch.Tensor, x_v: torch.Tensor, dst: List[int], B: int, npg: int):
        d = torch.tensor(dst, dtype=torch.int32).to(self.device, non_blocking=True)
        f = _fn("zs_kv_append_pages")
        for pool, x in ((self.k, x_k), (self.v, x_v)):
            check(f(_stream(), C.byref(pool.st), x.data_ptr(), B, npg, self.Hkv, D_HEAD, d.data_ptr(),
                    self.err.data_ptr()), "zs_kv_append_pages")

    def _new_block(self, seq: int) -> int:
        if len(self.blocks[seq]) >= self.max_blocks:
            raise RuntimeError(f"sequence {seq} exceeds {self.max_blocks * 64} tokens")
        blk = self.alloc.alloc()
        self.block_table[seq, len(self.blocks[seq])] = blk
        self.blocks[seq].append(blk)
        return blk

    def prefill(self, seq: int, k: torch.Tensor, v: torch.Tensor):
        """Start sequence `seq` with the prompt's K and V, [T, Hkv, 128] bf16."""
        if self.lengths[seq] or self.blocks[seq]:
            raise RuntimeError(f"sequence {seq} is in use; free it first")
        T = k.shape[0]
        if k.shape != (T, self.Hkv, D_HEAD) or v.shape != k.shape:
            raise ValueError("k and v must be [T, num_kv_heads, 128]")
        n = T // 64
        if n:
            dst = []
            for j in range(n):
                blk = self._new_block(seq)
                dst += [blk * self.Hkv + h for h in range(self.Hkv)]
            self._append(k[: 64 * n].contiguous(), v[: 64 * n].contiguous(), dst, 1, n)
        r = T - 64 * n
        if r:
            self.tail_k[seq, :r] = k[64 * n:]
            self.tail_v[seq, :r] = v[64 * n:]
        self.lengths[seq] = T
        self.seqlens[seq] = T

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor):
        """Append one token to each of sequences 0 .. B-1 (k_new, v_new:
        [B, Hkv, 128] bf16). Tail pages that become full are compressed into
        new blocks in one launch."""
        B = k_new.shape[0]
        if k_new.shape != (B, self.Hkv, D_HEAD) or v_new.shape != k_new.shape or B > self.max_batch:
            raise ValueError("k_new and v_new must be [B, num_kv_heads, 128] with B <= max_batch")
        pos = [self.lengths[b] % 64 for b in range(B)]
        idx_b = torch.arange(B, device=self.device)
        idx_t = torch.tensor(pos, dtype=torch.long).to(self.device, non_blocking=True)
        self.tail_k[idx_b, idx_t] = k_new
        self.tail_v[idx_b, idx_t] = v_new
        full = [b for b in range(B) if pos[b] == 63]
        dst = [-1] * (B * self.Hkv)
        for b in full:
            blk = self._new_block(b)
            for h in range(self.Hkv):
                dst[b * self.Hkv + h] = blk * self.Hkv + h
        if full:
            self._append(self.tail_k[:B], self.tail_v[:B], dst, B, 1)
        for b in range(B):
            self.lengths[b] += 1
        self.seqlens[:B] += 1

    def free(self, seq: int):
        self.alloc.free(self.blocks[seq])
        self.blocks[seq] = []
        self.lengths[seq] = 0
        self.seqlens[seq] = 0

    # ----------------------------------------------------------------- reads
    def attention(self, q: torch.Tensor, softmax_scale: Optional[float] = None, num_splits: int = 0,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Decode attention of q [B, Hq, 128] over sequences 0 .. B-1."""
        B, Hq, Dq = q.shape
        if Dq != D_HEAD or B > self.max_batch or Hq % self.Hkv:
            raise ValueError("q must be [B, Hq, 128] with Hq a multiple of num_kv_heads")
        scale = softmax_scale if softmax_scale is not None else D_HEAD ** -0.5
        max_len = max(self.lengths[:B]) if B else 0
        pages = (max_len + 63) // 64
        splits = num_splits if num_splits > 0 else _fn("zs_decode_attention_default_splits")(B, self.Hkv, 64 * pages)
        splits = max(1, min(splits, max(1, pages)))
        nbytes = _fn("zs_decode_attention_workspace_bytes")(B, Hq, self.Hkv, splits)
        ws = torch.empty(max(nbytes // 4, 1), dtype=torch.float32, device=self.device)
        if out is None:
            out = torch.empty_like(q)
        used = C.c_int(0)
        check(_fn("zs_decode_attention_paged")(
            _stream(), q.data_ptr(), C.byref(self.k.st), C.byref(self.v.st), self.block_table.data_ptr(),
            self.max_blocks, self.seqlens.data_ptr(), self.tail_k.data_ptr(), self.tail_v.data_ptr(), B, Hq,
            self.Hkv, D_HEAD, max_len, float(scale), splits, ws.data_ptr(), ws.numel() * 4, out.data_ptr(),
            C.byref(used), self.err.data_ptr()), "zs_decode_attention_paged")
        return out

    def check_errors(self) -> int:
        """Error bits recorded by the kernels (synchronises): 1 = a wait timed
        out, 2 = a page did not fit in the stream pools or an index was out of
        range."""
        return int(self.err.item())

    def dense(self, seq: int):
        """Dense [T, Hkv, 128] K and V of a sequence, decoded from the pools
        (for checks; uses zs_decompress on each page)."""
        from .codec import Compressed, decompress
        T = self.lengths[seq]
        ks, vs = [], []
        for blk in self.blocks[seq]:
            for pool, acc in ((self.k, ks), (self.v, vs)):
                page = torch.empty(self.Hkv, 64, D_HEAD, dtype=torch.bfloat16, device=self.device)
                offs = pool.page_off.view(-1, 6).cpu()
                for h in range(self.Hkv):
                    P = blk * self.Hkv + h
                    o = offs[P].tolist()
                    c = Compressed(pool.sm[o[0]:o[4] + 16], pool.full[o[1]:o[5] + 8],
                                   pool.b[0][P * 128:(P + 1) * 128], pool.b[1][P * 128:(P + 1) * 128],
                                   pool.b[2][P * 128:(P + 1) * 128], None, pool.mt_off[P * 16:(P + 1) * 16],
                                   torch.tensor([0, 0, o[2] - o[0], o[3] - o[1], o[4] - o[0], o[5] - o[1]],
                                                dtype=torch.int32, device=self.device),
                                   64, D_HEAD, 4096, 4096, pool.start_exp, o[4] - o[0], o[5] - o[1])
                    decompress(c, page[h])
                acc.append(page.permute(1, 0, 2))
        r = T % 64
        k = torch.cat(ks + [self.tail_k[seq, :r]]) if ks or r else self.tail_k[seq, :0]
        v = torch.cat(vs + [self.tail_v[seq, :r]]) if vs or r else self.tail_v[seq, :0]
        return k, v
