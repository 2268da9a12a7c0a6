"""Compressed-KV decode attention (torch-facing).

Mirrors the ZipServ decode path of the reference:
  * pad_kv_by_kv_head  -> kernel_benchmark/bench_zipserv_decode_attention.py:347
                          pad_batched_kv_prefix_by_kv_head ([B,T,Hkv,D] -> head-major 2-D)
  * compress_kv        -> the ext's compress_zipserv on that padded matrix
  * decode_attention   -> FA flash_attn_with_kvcache(q, ..., zipserv_k=, zipserv_v=,
                          zipserv_num_heads_k=) (FA flash_attn_interface.py:1592-1754)
  * flash_attn_with_kvcache -> the same call signature subset, taking the
                          reference's descriptor dicts (FA flash_attn_interface.py:23-36)
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Optional

import torch

from ._lib import check, lib
from .codec import Compressed, compress

_FIELDS = ("sign_mantissa", "compressed_full", "bitmap1", "bitmap2", "bitmap3", "tile_offsets_median",
           "tile_offsets_global")


def pad_kv_by_kv_head(x: torch.Tensor):
    """[B, T, Hkv, D] -> ([B*Hkv*T_pad, D_pad] zero padded, rows, T_pad)."""
    B, T, Hkv, D = x.shape
    t_pad = (T + 63) // 64 * 64
    d_pad = (D + 63) // 64 * 64
    out = torch.zeros((B, Hkv, t_pad, d_pad), dtype=x.dtype, device=x.device)
    out[:, :, :T, :D] = x.permute(0, 2, 1, 3)
    return out.view(B * Hkv * t_pad, d_pad), B * Hkv * t_pad, t_pad


def pad_kv_token_major(x: torch.Tensor):
    """[B, T, Hkv, D] -> ([B*T_pad*Hkv, D] zero padded, T_pad): the reference's
    token-major layout (row (b * T_pad + t) * Hkv + h; FA flash_api.cpp:1512-1520,
    layout id 1), T padded to a multiple of 64 so the rows form whole tiles."""
    B, T, Hkv, D = x.shape
    if 64 % Hkv or D % 64:   # FA flash_api.cpp:1514-1520
        raise ValueError("token-major layout needs Hkv dividing 64 and D a multiple of 64")
    t_pad = (T + 63) // 64 * 64
    out = torch.zeros((B, t_pad, Hkv, D), dtype=x.dtype, device=x.device)
    out[:, :T] = x
    return out.view(B * t_pad * Hkv, D), t_pad


def compress_kv(x: torch.Tensor, rule: str = "ext", layout: str = "by_kv_head") -> Compressed:
    """Compress a [B, T, Hkv, D] K or V cache: in the head-major 64-token page
    layout (default), or in the token-major layout (layout="token_major")."""
    if layout == "token_major":
        flat, _ = pad_kv_token_major(x)
    elif layout == "by_kv_head":
        flat, _, _ = pad_kv_by_kv_head(x)
    else:
        raise ValueError(f"unknown layout {layout!r}")
    return compress(flat, rule=rule)


def decode_attention_dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache_seqlens: torch.Tensor,
                           softmax_scale: Optional[float] = None, num_splits: int = 0,
                           max_seqlen: Optional[int] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The decode-attention kernel on an uncompressed token-major cache:
    q [B, Hq, D] (or [B, 1, Hq, D]), k / v [B, T_rows, Hkv, D] bf16 with
    T_rows % 64 == 0 (every page read dense)."""
    squeeze = q.dim() == 4
    q3 = (q.reshape(q.shape[0], q.shape[-2], q.shape[-1]) if squeeze else q).contiguous()
    B, Hq, D = q3.shape
    if k.shape != v.shape or k.dim() != 4 or k.shape[0] != B or k.dtype != torch.bfloat16:
        raise ValueError("k / v must be bf16 [B, T_rows, Hkv, D] tensors of the same shape")
    t_rows, hk = k.shape[1], k.shape[2]
    k, v = k.contiguous(), v.contiguous()
    seq = cache_seqlens.to(device=q3.device, dtype=torch.int32).contiguous()
    max_seqlen = t_rows if max_seqlen is None else min(max_seqlen, t_rows)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    L = lib()
    splits = num_splits if num_splits > 0 else L.zs_decode_attention_default_splits(B, hk, max_seqlen)
    ws_bytes = L.zs_decode_attention_workspace_bytes(B, Hq, hk, splits)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=q3.device)
    if out is None:
        out = torch.empty_like(q3)
    check(L.zs_decode_attention_dense(torch.cuda.current_stream().cuda_stream, q3.data_ptr(), k.data_ptr(),
                                      v.data_ptr(), seq.data_ptr(), B, Hq, hk, D, t_rows, max_seqlen, scale, splits,
                                      ws.data_ptr(), ws_bytes, out.data_ptr(), None, None),
          "zs_decode_attention_dense")
    return out.view(q.shape) if squeeze else out


def _ptrs_meta(c: Compressed):
    ptrs = (C.c_void_p * 7)(*[getattr(c, f).data_ptr() for f in _FIELDS])
    meta = (C.c_int * 5)(c.rows, c.cols, c.max_high_freq_count, c.max_full_count, c.start_exp)
    return ptrs, meta


def decode_attention(q: torch.Tensor, k: Compressed, v: Compressed, cache_seqlens: torch.Tensor,
                     num_heads_k: int, softmax_scale: Optional[float] = None, num_splits: int = 0,
                     max_seqlen: Optional[int] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q: [B, Hq, D] (or [B, 1, Hq, D]) bf16; returns the same shape."""
    squeeze = q.dim() == 4
    q3 = q.reshape(q.shape[0], q.shape[-2], q.shape[-1]) if squeeze else q
    if q3.dtype != torch.bfloat16 or not q3.is_cuda:
        raise ValueError("q must be a bf16 CUDA tensor")
    q3 = q3.contiguous()
    B, Hq, D = q3.shape
    if Hq % num_heads_k:
        raise ValueError("num_heads must be a multiple of num_heads_k")
    if k.rows % (B * num_heads_k) or k.rows != v.rows or k.cols != v.cols:
        raise ValueError("K/V row count must be B * num_heads_k * T_pad and agree")
    t_pad = k.rows // (B * num_heads_k)
    seq = cache_seqlens.to(device=q3.device, dtype=torch.int32).contiguous()
    # the bound only sizes the split-KV grid; without one the padded length is
    # used, so the call never reads cache_seqlens back to the host
    max_seqlen = t_pad if max_seqlen is None else min(max_seqlen, t_pad)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    L = lib()
    splits = num_splits if num_splits > 0 else L.zs_decode_attention_default_splits(B, num_heads_k, max_seqlen)
    ws_bytes = L.zs_decode_attention_workspace_bytes(B, Hq, num_heads_k, splits)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=q3.device)
    if out is None:
        out = torch.empty_like(q3)
    kp, km = _ptrs_meta(k)
    vp, vm = _ptrs_meta(v)
    used = C.c_int(0)
    check(L.zs_decode_attention(torch.cuda.current_stream().cuda_stream, q3.data_ptr(), kp, km, vp, vm,
                                seq.data_ptr(), B, Hq, num_heads_k, D, t_pad, max_seqlen, scale, splits,
                                ws.data_ptr(), ws_bytes, out.data_ptr(), C.byref(used), None),
          "zs_decode_attention")
    return out.view(q.shape) if squeeze else out


def _as_compressed(desc, device) -> Compressed:
    if isinstance(desc, Compressed):
        return desc
    if isinstance(desc, dict):
        vals = {f: desc[f] for f in _FIELDS}
        rows, cols = int(desc["rows"]), int(desc["cols"])
        mh, mf, se = int(desc["max_high_freq_count"]), int(desc["max_full_count"]), int(desc["start_exp"])
    else:  # sequence in the reference's field order (FA flash_attn_interface.py:23-36)
        vals = dict(zip(_FIELDS, desc[:7]))
        rows, cols, mh, mf, se = (int(x) for x in desc[7:12])
    for f, t in vals.items():
        if not isinstance(t, torch.Tensor) or t.device != device:
            raise ValueError(f"{f} must be a tensor on {device}")
    return Compressed(vals["sign_mantissa"], vals["compressed_full"], vals["bitmap1"], vals["bitmap2"],
                      vals["bitmap3"], None, vals["tile_offsets_median"], vals["tile_offsets_global"], rows, cols,
                      mh, mf, se & 0xFF, 0, 0)


def flash_attn_with_kvcache(q, k_cache=None, v_cache=None, cache_seqlens=None, softmax_scale=None,
                            num_splits=0, zipserv_k=None, zipserv_v=None, zipserv_num_heads_k=None, **unused):
    """Decode-attention entry with the reference's ZipServ keyword arguments.

    q is [B, 1, Hq, D]; zipserv_k / zipserv_v are descriptors as accepted by the
    reference (dict with the 12 fields, or a sequence in that order; layout
    "by_kv_head" or "token_major"). Only the compressed path is provided here."""
    if zipserv_k is None or zipserv_v is None:
        raise ValueError("zipserv_k and zipserv_v are required")
    layouts = {d.get("layout", "by_kv_head") if isinstance(d, dict) else "by_kv_head" for d in (zipserv_k, zipserv_v)}
    if len(layouts) != 1 or not layouts <= {"by_kv_head", "token_major", 0, 1}:
        raise ValueError("zipserv K and V must share one layout: by_kv_head (0) or token_major (1)")
    layout = layouts.pop()
    hk = zipserv_num_heads_k if zipserv_num_heads_k else (k_cache.shape[2] if k_cache is not None else 0)
    if not hk:
        raise ValueError("zipserv_num_heads_k must be provided")
    k = _as_compressed(zipserv_k, q.device)
    v = _as_compressed(zipserv_v, q.device)
    if layout in ("token_major", 1):
        # Token-major pages interleave the KV heads (a 64-row tile holds 64 / Hkv
        # tokens of every head), so the cache is expanded by the decompress
        # kernel and attended with every page read dense: two stages of this
        # library's kernels, where the reference decodes in its FA2 loop
        # (FA flash_fwd_kernel.h:325-430).
        B = q.shape[0]
        if 64 % hk:   # FA flash_api.cpp:1514-1520
            raise ValueError("token-major layout requires 64 % zipserv_num_heads_k == 0")
        if k.rows % (B * hk) or k.rows != v.rows or k.cols != v.cols:
            raise ValueError("token-major K/V rows must be B * T_pad * Hkv and agree")
        t_rows = k.rows // (B * hk)
        from .codec import decompress
        kd = decompress(k).view(B, t_rows, hk, k.cols)
        vd = decompress(v).view(B, t_rows, hk, v.cols)
        if cache_seqlens is None:
            cache_seqlens = torch.full((B,), t_rows, dtype=torch.int32, device=q.device)
        elif not isinstance(cache_seqlens, torch.Tensor):
            cache_seqlens = torch.full((B,), int(cache_seqlens), dtype=torch.int32, device=q.device)
        return decode_attention_dense(q, kd, vd, cache_seqlens, softmax_scale, num_splits)
    if cache_seqlens is None:
        cache_seqlens = torch.full((q.shape[0],), k.rows // (q.shape[0] * hk), dtype=torch.int32, device=q.device)
    elif not isinstance(cache_seqlens, torch.Tensor):
        cache_seqlens = torch.full((q.shape[0],), int(cache_seqlens), dtype=torch.int32, device=q.device)
    return decode_attention(q, k, v, cache_seqlens, hk, softmax_scale, num_splits)
