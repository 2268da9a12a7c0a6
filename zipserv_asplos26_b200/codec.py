"""Torch-facing TCA-TBE codec and ZipGEMM on the CUDA library.

Device memory comes from torch; all kernels run on torch's *current* CUDA
stream. Functions mirror the reference entry points:
  compress()    -> kernel_benchmark/zipserv_decode_attention_ext.cu:157 compress_zipserv_cuda
                   (GPU window analysis + csrc/L_API.cu:1355 encoder)
  decompress()  -> csrc/L_API.cu:234 BF16TripleBitmap_Decompress_API
  zipgemm()     -> csrc/L_API.cu:119 BF16TripleBitmap_MM_API
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch

from ._lib import check, lib

RULES = {"host": 0, "ext": 1}


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


@dataclass
class Compressed:
    """A TCA-TBE compressed rows x cols bf16 matrix resident on one GPU.

    Field names follow the reference ext / FlashAttention descriptor
    (flash_attn_interface.py:23-36)."""

    sign_mantissa: torch.Tensor        # uint8  [>= total_hf]
    compressed_full: torch.Tensor      # bf16   [>= total_full]
    bitmap1: torch.Tensor              # uint64 [#ST]
    bitmap2: torch.Tensor
    bitmap3: torch.Tensor
    tile_offsets: torch.Tensor         # int32  [2 * #ST]  per small tile (hf, fallback) counts
    tile_offsets_median: torch.Tensor  # int32  [2 * #MT]
    tile_offsets_global: torch.Tensor  # int32  [2 * (#GT + 1)]
    rows: int
    cols: int
    max_high_freq_count: int
    max_full_count: int
    start_exp: int
    total_hf: int
    total_full: int
    top: list = field(default_factory=list)

    @property
    def num_global_tiles(self) -> int:
        return (self.rows // 64) * (self.cols // 64)

    def compressed_bytes(self) -> int:
        """Streams + bitmaps + median/global offsets (test_mm.cu:696-703 definition)."""
        nst = self.rows * self.cols // 64
        nmt = nst // 16
        return (self.total_hf + 2 * self.total_full + 24 * nst + 8 * nmt
                + 8 * (self.num_global_tiles + 1))

    def ext_compressed_bytes(self) -> int:
        """The torch extension's definition (ext.cu:23-33): adds ST offsets and 28 bytes."""
        nst = self.rows * self.cols // 64
        return self.compressed_bytes() + 8 * nst + 28

    def descriptor(self, layout: str = "by_kv_head") -> dict:
        return dict(sign_mantissa=self.sign_mantissa, compressed_full=self.compressed_full,
                    bitmap1=self.bitmap1, bitmap2=self.bitmap2, bitmap3=self.bitmap3,
                    tile_offsets_median=self.tile_offsets_median,
                    tile_offsets_global=self.tile_offsets_global, rows=self.rows, cols=self.cols,
                    max_high_freq_count=self.max_high_freq_count,
                    max_full_count=self.max_full_count, start_exp=self.start_exp, layout=layout)


def _check_2d_bf16(x: torch.Tensor, name: str):
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError(f"{name} must be a contiguous 2-D bfloat16 tensor")


def analyze_exponents(w: torch.Tensor, rule: str = "host") -> torch.Tensor:
    """7-exponent window on the GPU (int32[7] device tensor, stream ordered)."""
    L = lib()
    scratch = torch.empty(L.zs_analyze_scratch_bytes(), dtype=torch.uint8, device=w.device)
    top = torch.empty(7, dtype=torch.int32, device=w.device)
    check(L.zs_analyze_exponents(_stream(), w.data_ptr(), w.numel(), RULES[rule], scratch.data_ptr(),
                                 top.data_ptr()), "zs_analyze_exponents")
    return top


def compress(w: torch.Tensor, rule: str = "host", top: Optional[torch.Tensor] = None,
             trim: bool = False) -> Compressed:
    """Compress a 2-D bf16 CUDA tensor (rows, cols multiples of 64).

    Like the reference extension this synchronises the current stream once to
    read the stream lengths and maxima back to the host."""
    _check_2d_bf16(w, "w")
    M, K = w.shape
    if M % 64 or K % 64:
        raise ValueError("rows and cols must be multiples of 64")
    L = lib()
    dev = w.device
    ngt = (M // 64) * (K // 64)
    nst = M * K // 64
    nmt = nst // 16
    if top is None:
        top = analyze_exponents(w, rule)
    top = top.to(device=dev, dtype=torch.int32).contiguous()
    sm = torch.empty(M * K + 16 * ngt, dtype=torch.uint8, device=dev)
    full = torch.empty(M * K + 8 * ngt, dtype=torch.bfloat16, device=dev)
    b = [torch.empty(nst, dtype=torch.uint64, device=dev) for _ in range(3)]
    st = torch.empty(2 * nst, dtype=torch.int32, device=dev)
    mt = torch.empty(2 * nmt, dtype=torch.int32, device=dev)
    gt = torch.empty(2 * (ngt + 1), dtype=torch.int32, device=dev)
    scratch = torch.empty(L.zs_encode_scratch_bytes(M, K), dtype=torch.uint8, device=dev)
    scal = torch.empty(4, dtype=torch.int32, device=dev)
    check(L.zs_encode(_stream(), w.data_ptr(), M, K, top.data_ptr(), sm.data_ptr(), full.data_ptr(),
                      b[0].data_ptr(), b[1].data_ptr(), b[2].data_ptr(), st.data_ptr(), mt.data_ptr(),
                      gt.data_ptr(), scratch.data_ptr(), scal.data_ptr()), "zs_encode")
    host = torch.cat([scal, top]).cpu().tolist()  # synchronises the stream
    max_hf, max_full, thf, tfull = host[:4]
    topl = host[4:]
    if trim:
        sm = sm[: max(thf, 16)].clone()
        full = full[: max(tfull, 8)].clone()
    return Compressed(sm, full, b[0], b[1], b[2], st, mt, gt, M, K, max_hf, max_full,
                      (topl[0] - 1) & 0xFF, thf, tfull, topl)


def compress_host(w: torch.Tensor, rule: str = "host") -> Compressed:
    """Compress a 2-D bf16 CPU tensor with the library's multi-threaded host
    encoder (csrc/L_API.cu:559 InitBF16MatrixTripleBitmap_Reuse semantics,
    byte-identical to the GPU encoder); the result's tensors live on the CPU,
    trimmed to their valid lengths."""
    if w.is_cuda or w.dtype != torch.bfloat16 or w.dim() != 2:
        raise ValueError("w must be a 2-D bfloat16 CPU tensor")
    w = w.contiguous()
    M, K = w.shape
    if M % 64 or K % 64:
        raise ValueError("rows and cols must be multiples of 64")
    L = lib()
    ngt = (M // 64) * (K // 64)
    nst = M * K // 64
    nmt = nst // 16
    top = torch.empty(7, dtype=torch.int32)
    check(L.zs_analyze_exponents_host(w.data_ptr(), w.numel(), RULES[rule], top.data_ptr()),
          "zs_analyze_exponents_host")
    sm = torch.empty(M * K + 16 * ngt, dtype=torch.uint8)
    full = torch.empty(M * K + 8 * ngt, dtype=torch.bfloat16)
    b = [torch.empty(nst, dtype=torch.uint64) for _ in range(3)]
    st = torch.empty(2 * nst, dtype=torch.int32)
    mt = torch.empty(2 * nmt, dtype=torch.int32)
    gt = torch.empty(2 * (ngt + 1), dtype=torch.int32)
    scal = torch.empty(4, dtype=torch.int32)
    check(L.zs_encode_host(w.data_ptr(), M, K, top.data_ptr(), sm.data_ptr(), full.data_ptr(), b[0].data_ptr(),
                           b[1].data_ptr(), b[2].data_ptr(), st.data_ptr(), mt.data_ptr(), gt.data_ptr(),
                           scal.data_ptr()), "zs_encode_host")
    max_hf, max_full, thf, tfull = scal.tolist()
    topl = top.tolist()
    return Compressed(sm[: max(thf, 16)].clone(), full[: max(tfull, 8)].clone(), b[0], b[1], b[2], st, mt, gt, M,
                      K, max_hf, max_full, (topl[0] - 1) & 0xFF, thf, tfull, topl)


def to_device(c: Compressed, device) -> Compressed:
    """Copy a compressed matrix's arrays to `device` (the streams keep 16 bytes of
    read slack past their valid length, as the GPU encoder's buffers do)."""
    def pad(t, extra):
        out = torch.zeros(t.numel() + extra, dtype=t.dtype)
        out[: t.numel()] = t
        return out.to(device)
    return Compressed(pad(c.sign_mantissa, 16), pad(c.compressed_full, 8), c.bitmap1.to(device),
                      c.bitmap2.to(device), c.bitmap3.to(device),
                      None if c.tile_offsets is None else c.tile_offsets.to(device),
                      c.tile_offsets_median.to(device), c.tile_offsets_global.to(device), c.rows, c.cols,
                      c.max_high_freq_count, c.max_full_count, c.start_exp, c.total_hf, c.total_full, list(c.top))


def decompress(c: Compressed, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(c.rows, c.cols, dtype=torch.bfloat16, device=c.bitmap1.device)
    _check_2d_bf16(out, "out")
    if tuple(out.shape) != (c.rows, c.cols):
        raise ValueError("output shape must equal (rows, cols)")
    check(lib().zs_decompress(_stream(), c.sign_mantissa.data_ptr(), c.compressed_full.data_ptr(),
                              c.bitmap1.data_ptr(), c.bitmap2.data_ptr(), c.bitmap3.data_ptr(),
                              c.tile_offsets_median.data_ptr(), c.tile_offsets_global.data_ptr(),
                              c.max_high_freq_count, c.max_full_count, c.start_exp, out.data_ptr(),
                              c.rows, c.cols, None), "zs_decompress")
    return out


def zipgemm(c: Compressed, x: torch.Tensor, out: Optional[torch.Tensor] = None,
            split_k: int = 1) -> torch.Tensor:
    """Y = W @ x^T for token-major x [N, K]; returns out [N, M] (== column-major M x N)."""
    _check_2d_bf16(x, "x")
    N, K = x.shape
    if K != c.cols:
        raise ValueError("x.shape[1] must equal the compressed matrix's cols")
    if out is None:
        out = torch.empty(N, c.rows, dtype=torch.bfloat16, device=x.device)
    _check_2d_bf16(out, "out")
    if tuple(out.shape) != (N, c.rows):
        raise ValueError("out must be [N, rows]")
    check(lib().zs_zipgemm(_stream(), c.sign_mantissa.data_ptr(), c.compressed_full.data_ptr(),
                           c.bitmap1.data_ptr(), c.bitmap2.data_ptr(), c.bitmap3.data_ptr(),
                           c.tile_offsets_median.data_ptr(), c.tile_offsets_global.data_ptr(),
                           c.max_high_freq_count, c.max_full_count, c.start_exp, x.data_ptr(),
                           out.data_ptr(), c.rows, N, K, split_k, None), "zs_zipgemm")
    return out
