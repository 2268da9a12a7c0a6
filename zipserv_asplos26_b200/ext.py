"""Drop-in for the reference torch extension `zipserv_decode_attention_ext`
(kernel_benchmark/zipserv_decode_attention_ext.cpp:177-181): same function
names, argument meaning, return values and input checks, on the B200 library.

    compress_zipserv(input, logical_rows, logical_cols) -> [sign_mantissa,
        compressed_full, bitmap1, bitmap2, bitmap3, tile_offsets_median,
        tile_offsets_global, meta]                       (ext.cu:157-265)
    decompress_zipserv(sign_mantissa, ..., rows, cols, max_hf, max_full, start_exp)
    decompress_zipserv_into(output, sign_mantissa, ..., start_exp)

meta is int64[11] = (rows, cols, logical_rows, logical_cols, max_high_freq_count,
max_full_count, start_exp, total_hf, total_full, num_global_tiles,
compressed_bytes) with compressed_bytes in the extension's definition
(ext.cu:23-33). As in the reference, the window is chosen with the extension's
GPU rule (ext.cu:65-133) and the stream tensors are allocated at full size
(rows * cols); the valid lengths are in meta. Work is ordered on torch's
current CUDA stream (the reference uses the default stream)."""
from __future__ import annotations

from typing import List

import torch

from ._lib import check, lib
from .codec import Compressed, compress

_NAMES = ("sign_mantissa", "compressed_full", "bitmap1", "bitmap2", "bitmap3", "tile_offsets_median",
          "tile_offsets_global")
_DTYPES = (torch.uint8, torch.bfloat16, torch.uint64, torch.uint64, torch.uint64, torch.int32, torch.int32)


def _check_cuda(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _check_compressed(tensors):
    for t, n, dt in zip(tensors, _NAMES, _DTYPES):
        _check_cuda(t, n)
        if t.dtype != dt:
            raise RuntimeError(f"{n} must be {str(dt).replace('torch.', '')}")


def compress_zipserv(input: torch.Tensor, logical_rows: int, logical_cols: int) -> List[torch.Tensor]:
    _check_cuda(input, "input")
    if input.dtype != torch.bfloat16:
        raise RuntimeError("input must be bfloat16")
    if input.dim() != 2:
        raise RuntimeError("input must be 2D")
    rows, cols = input.shape
    if rows % 64:
        raise RuntimeError("rows must be padded to a multiple of 64")
    if cols % 64:
        raise RuntimeError("cols must be padded to a multiple of 64")
    c = compress(input, rule="ext")
    numel = rows * cols
    sm = torch.zeros(numel, dtype=torch.uint8, device=input.device)
    full = torch.zeros(numel, dtype=torch.bfloat16, device=input.device)
    sm[: c.total_hf] = c.sign_mantissa[: c.total_hf]
    full[: c.total_full] = c.compressed_full[: c.total_full]
    meta = torch.tensor([rows, cols, int(logical_rows), int(logical_cols), c.max_high_freq_count, c.max_full_count,
                         (c.top[0] - 1), c.total_hf, c.total_full, c.num_global_tiles, c.ext_compressed_bytes()],
                        dtype=torch.int64)
    return [sm, full, c.bitmap1, c.bitmap2, c.bitmap3, c.tile_offsets_median, c.tile_offsets_global, meta]


def decompress_zipserv_into(output: torch.Tensor, sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3,
                            tile_offsets_median, tile_offsets_global, rows: int, cols: int,
                            max_high_freq_count: int, max_full_count: int, start_exp: int) -> torch.Tensor:
    _check_cuda(output, "output")
    if output.dtype != torch.bfloat16:
        raise RuntimeError("output must be bfloat16")
    if output.dim() != 2:
        raise RuntimeError("output must be 2D")
    if output.size(0) != rows:
        raise RuntimeError("output rows must match rows")
    if output.size(1) != cols:
        raise RuntimeError("output cols must match cols")
    ts = (sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3, tile_offsets_median, tile_offsets_global)
    _check_compressed(ts)
    check(lib().zs_decompress(torch.cuda.current_stream().cuda_stream, *[t.data_ptr() for t in ts],
                              int(max_high_freq_count), int(max_full_count), int(start_exp) & 0xFF,
                              output.data_ptr(), int(rows), int(cols), None), "decompress_zipserv_into")
    return output


def decompress_zipserv(sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3, tile_offsets_median,
                       tile_offsets_global, rows: int, cols: int, max_high_freq_count: int, max_full_count: int,
                       start_exp: int) -> torch.Tensor:
    _check_compressed((sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3, tile_offsets_median,
                       tile_offsets_global))
    out = torch.empty((int(rows), int(cols)), dtype=torch.bfloat16, device=compressed_full.device)
    return decompress_zipserv_into(out, sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3,
                                   tile_offsets_median, tile_offsets_global, rows, cols, max_high_freq_count,
                                   max_full_count, start_exp)


def from_ext_outputs(outs) -> Compressed:
    """Wrap compress_zipserv's 8 outputs as a Compressed (for zipgemm / attention)."""
    sm, full, b1, b2, b3, mt, gt, meta = outs
    m = meta.tolist()
    return Compressed(sm, full, b1, b2, b3, None, mt, gt, m[0], m[1], m[4], m[5], m[6] & 0xFF, m[7], m[8])
