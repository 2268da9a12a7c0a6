"""Save and load TCA-TBE compressed matrices (file format version 1).

The container is written and read by the library's C ABI (`zs_tcatbe_save`,
`zs_tcatbe_read_info`, `zs_tcatbe_load` in include/zipserv_b200.h), so C and
Python callers share one implementation. The reference keeps no serialised
compressed form (its benchmarks re-encode the dense checkpoint at start-up,
kernel_benchmark/bench_zipserv_gemm_sweep.cu:290-345); this lets a server load
compressed weights directly and copy only compressed bytes to the GPU.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Union

import torch

from ._lib import ZipServError, lib
from .codec import Compressed


class ZsTcatbeInfo(C.Structure):
    _fields_ = [("rows", C.c_int64), ("cols", C.c_int64), ("start_exp", C.c_int32), ("max_hf", C.c_int32),
                ("max_full", C.c_int32), ("top", C.c_int32 * 7), ("total_hf", C.c_int64),
                ("total_full", C.c_int64), ("has_st_counts", C.c_int32)]


_P = C.c_void_p
_SIGS = {
    "zs_tcatbe_save": ([C.c_char_p, C.POINTER(ZsTcatbeInfo)] + [_P] * 8, C.c_int),
    "zs_tcatbe_read_info": ([C.c_char_p, C.POINTER(ZsTcatbeInfo)], C.c_int),
    "zs_tcatbe_load": ([C.c_char_p, C.POINTER(ZsTcatbeInfo)] + [_P] * 8, C.c_int),
}


def _fn(name):
    f = getattr(lib(), name)
    f.argtypes, f.restype = _SIGS[name]
    return f


def _check(status: int, what: str, path):
    if status != 0:
        reason = {301: "cannot open file", 999: "short read or write",
                  1: "invalid arguments or not a valid TCA-TBE file (magic, version, sizes or checksum)"}
        raise ZipServError(f"{what}({path!r}) failed with status {status}: {reason.get(status, 'error')}")


def _host(t: Optional[torch.Tensor], n: int, dtype) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = t.reshape(-1)[:n]
    return t.to("cpu").view(dtype).contiguous()


def save(c: Compressed, path: Union[str, os.PathLike]) -> None:
    """Write `c` (on any device) to `path`. The small-tile counts are stored
    when `c.tile_offsets` is present; no kernel reads them."""
    rows, cols = c.rows, c.cols
    nst = rows * cols // 64
    nmt, ngt = nst // 16, nst // 64
    sm = _host(c.sign_mantissa, c.total_hf, torch.uint8)
    full = _host(c.compressed_full, c.total_full, torch.int16)
    b = [_host(x, nst, torch.int64) for x in (c.bitmap1, c.bitmap2, c.bitmap3)]
    st = _host(c.tile_offsets, 2 * nst, torch.int32)
    mt = _host(c.tile_offsets_median, 2 * nmt, torch.int32)
    gt = _host(c.tile_offsets_global, 2 * (ngt + 1), torch.int32)
    info = ZsTcatbeInfo(rows=rows, cols=cols, start_exp=c.start_exp, max_hf=c.max_high_freq_count,
                        max_full=c.max_full_count, total_hf=c.total_hf, total_full=c.total_full,
                        has_st_counts=1 if st is not None and st.numel() == 2 * nst else 0)
    top = list(c.top) + [0] * (7 - len(c.top))
    for i in range(7):
        info.top[i] = int(top[i])
    ptr = lambda t: None if t is None or t.numel() == 0 else t.data_ptr()
    _check(_fn("zs_tcatbe_save")(os.fsencode(path), C.byref(info), ptr(sm), ptr(full), ptr(b[0]), ptr(b[1]),
                                 ptr(b[2]), ptr(st) if info.has_st_counts else None, ptr(mt), ptr(gt)),
           "zs_tcatbe_save", path)


def read_info(path: Union[str, os.PathLike]) -> dict:
    info = ZsTcatbeInfo()
    _check(_fn("zs_tcatbe_read_info")(os.fsencode(path), C.byref(info)), "zs_tcatbe_read_info", path)
    return dict(rows=info.rows, cols=info.cols, start_exp=info.start_exp, max_hf=info.max_hf,
                max_full=info.max_full, top=list(info.top), total_hf=info.total_hf, total_full=info.total_full,
                has_st_counts=bool(info.has_st_counts))


def load(path: Union[str, os.PathLike], device: Union[str, torch.device, None] = None,
         with_st_counts: bool = False) -> Compressed:
    """Read a compressed matrix. With `device` set to a CUDA device the arrays
    are read into pinned host memory and copied on the current stream; the
    streams keep the 16 bytes (sign/mantissa) and 8 elements (fallback) of
    read slack the GPU decoders expect past their valid length."""
    info = ZsTcatbeInfo()
    p = os.fsencode(path)
    _check(_fn("zs_tcatbe_read_info")(p, C.byref(info)), "zs_tcatbe_read_info", path)
    rows, cols = int(info.rows), int(info.cols)
    nst = rows * cols // 64
    nmt, ngt = nst // 16, nst // 64
    dev = torch.device(device) if device is not None else torch.device("cpu")
    pin = dev.type == "cuda"
    mk = lambda n, dt: torch.zeros(n, dtype=dt, pin_memory=pin)
    sm = mk(int(info.total_hf) + 16, torch.uint8)
    full = mk(int(info.total_full) + 8, torch.bfloat16)
    b = [mk(nst, torch.uint64) for _ in range(3)]
    keep_st = with_st_counts and bool(info.has_st_counts)
    st = mk(2 * nst, torch.int32) if keep_st else None
    mt = mk(2 * nmt, torch.int32)
    gt = mk(2 * (ngt + 1), torch.int32)
    _check(_fn("zs_tcatbe_load")(p, C.byref(info), sm.data_ptr(), full.data_ptr(), b[0].data_ptr(),
                                 b[1].data_ptr(), b[2].data_ptr(), None if st is None else st.data_ptr(),
                                 mt.data_ptr(), gt.data_ptr()), "zs_tcatbe_load", path)
    if dev.type != "cpu":
        mv = lambda t: None if t is None else t.to(dev, non_blocking=True)
        sm, full, st, mt, gt = mv(sm), mv(full), mv(st), mv(mt), mv(gt)
        b = [mv(x) for x in b]
    return Compressed(sm, full, b[0], b[1], b[2], st, mt, gt, rows, cols, int(info.max_hf), int(info.max_full),
                      int(info.start_exp), int(info.total_hf), int(info.total_full), list(info.top))
