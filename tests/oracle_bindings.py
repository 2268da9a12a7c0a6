"""Test-side ctypes bindings for the CPU oracle (oracle/lib/liboracle.so) and for
the reference library compiled from source (oracle/_ref/libzipserv_ref.so).

Test infrastructure only: the product package never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "lib", "liboracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libzipserv_ref.so")

_P = C.c_void_p


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


@dataclass
class Encoded:
    """The seven TCA-TBE streams plus scalars, trimmed to their valid length."""

    sign_mantissa: np.ndarray  # uint8 [total_hf]
    full: np.ndarray           # uint16 (bf16 bits) [total_full]
    bitmap1: np.ndarray        # uint64 [#ST]
    bitmap2: np.ndarray
    bitmap3: np.ndarray
    st_counts: np.ndarray      # int32 [2 * #ST]
    mt_offsets: np.ndarray     # int32 [2 * #MT]
    gt_offsets: np.ndarray     # int32 [2 * (#GT + 1)]
    max_hf: int
    max_full: int
    top: np.ndarray            # int32 [7]

    @property
    def start_exp(self) -> int:
        return (int(self.top[0]) - 1) & 0xFF

    @property
    def total_hf(self) -> int:
        return int(self.gt_offsets[-2])

    @property
    def total_full(self) -> int:
        return int(self.gt_offsets[-1])

    def compressed_bytes(self) -> int:
        """test_mm.cu:696-703 definition: streams + bitmaps + MT/GT offsets."""
        return (self.total_hf + 2 * self.total_full + 3 * 8 * self.bitmap1.size
                + 4 * self.mt_offsets.size + 4 * self.gt_offsets.size)


def _alloc(M: int, K: int):
    ngt = (M // 64) * (K // 64)
    nst = M * K // 64
    nmt = M * K // 1024
    return dict(
        sm=np.zeros(M * K + 16 * ngt + 64, np.uint8),
        full=np.zeros(M * K + 8 * ngt + 64, np.uint16),
        b1=np.zeros(nst, np.uint64), b2=np.zeros(nst, np.uint64), b3=np.zeros(nst, np.uint64),
        st=np.zeros(2 * nst, np.int32), mt=np.zeros(2 * nmt, np.int32),
        gt=np.zeros(2 * (ngt + 1), np.int32),
    )


def _trim(buf, max_hf, max_full, top) -> Encoded:
    gt = buf["gt"]
    return Encoded(buf["sm"][: gt[-2]].copy(), buf["full"][: gt[-1]].copy(), buf["b1"], buf["b2"],
                   buf["b3"], buf["st"], buf["mt"], gt, int(max_hf), int(max_full),
                   np.asarray(top, np.int32))


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        self.lib = C.CDLL(path)
        L = self.lib
        L.oracle_analyze_host.argtypes = [_P, C.c_int64, _P]
        L.oracle_analyze_ext.argtypes = [_P, C.c_int64, _P]
        L.oracle_encode.argtypes = [_P, C.c_int, C.c_int, _P] + [_P] * 8 + [_P] * 4
        L.oracle_encode.restype = C.c_int
        L.oracle_decode.argtypes = [_P, C.c_int64, _P, C.c_int64, _P, _P, _P, _P, C.c_int,
                                    C.c_int, C.c_int, _P]
        L.oracle_decode.restype = C.c_int
        L.oracle_gemm.argtypes = [_P, _P, C.c_int, C.c_int, C.c_int, _P]

    def analyze(self, a: np.ndarray, rule: str = "host") -> np.ndarray:
        a = np.ascontiguousarray(a, np.uint16)
        top = np.zeros(7, np.int32)
        fn = self.lib.oracle_analyze_host if rule == "host" else self.lib.oracle_analyze_ext
        fn(_ptr(a), a.size, _ptr(top))
        return top

    def encode(self, a: np.ndarray, top=None) -> Encoded:
        a = np.ascontiguousarray(a, np.uint16)
        M, K = a.shape
        if top is None:
            top = self.analyze(a)
        top = np.ascontiguousarray(top, np.int32)
        b = _alloc(M, K)
        s = np.zeros(4, np.int32)
        self.lib.oracle_encode(_ptr(a), M, K, _ptr(top), _ptr(b["sm"]), _ptr(b["full"]),
                               _ptr(b["b1"]), _ptr(b["b2"]), _ptr(b["b3"]), _ptr(b["st"]),
                               _ptr(b["mt"]), _ptr(b["gt"]), _ptr(s[0:]), _ptr(s[1:]),
                               _ptr(s[2:]), _ptr(s[3:]))
        return _trim(b, s[0], s[1], top)

    def decode(self, e: Encoded, M: int, K: int, start_exp=None) -> np.ndarray:
        out = np.zeros((M, K), np.uint16)
        se = e.start_exp if start_exp is None else start_exp
        sm = np.ascontiguousarray(e.sign_mantissa)
        fu = np.ascontiguousarray(e.full)
        r = self.lib.oracle_decode(_ptr(sm), sm.size, _ptr(fu), fu.size, _ptr(e.bitmap1),
                                   _ptr(e.bitmap2), _ptr(e.bitmap3), _ptr(e.gt_offsets), se, M, K,
                                   _ptr(out))
        if r != 0:
            raise ValueError("oracle_decode: stream index out of range")
        return out

    def gemm(self, w_bits: np.ndarray, x_bits: np.ndarray) -> np.ndarray:
        """C[n*M+m] = sum_k W[m,k] X[n,k] in double; returns float64 [N, M]."""
        w = np.ascontiguousarray(w_bits, np.uint16)
        x = np.ascontiguousarray(x_bits, np.uint16)
        M, K = w.shape
        N = x.shape[0]
        c = np.zeros((N, M), np.float64)
        self.lib.oracle_gemm(_ptr(w), _ptr(x), M, N, K, _ptr(c))
        return c


class Reference:
    """The reference's own host encoders, compiled from its sources."""

    def __init__(self, path: str = REF_SO):
        self.lib = C.CDLL(path)
        L = self.lib
        L.ref_analyze.argtypes = [_P, C.c_int, C.c_int, _P]
        L.ref_init_matrices.argtypes = [_P, _P, C.c_int, C.c_int, C.c_int, C.c_uint]
        L.ref_encode_scalar.argtypes = [_P, C.c_int, C.c_int, _P] + [_P] * 10
        L.ref_encode_scalar.restype = C.c_int
        for fn in (L.ref_encode_reuse, L.ref_encode_simd):
            fn.argtypes = [_P, C.c_int, C.c_int, _P] + [_P] * 12
            fn.restype = C.c_int
        L.ref_mm.argtypes = [_P] * 8 + [C.c_int] * 3 + [_P, _P, C.c_int, C.c_int, C.c_int, _P, C.c_int]
        L.ref_mm.restype = C.c_int
        L.ref_decompress.argtypes = [_P] * 8 + [C.c_int] * 3 + [_P, C.c_int, C.c_int]
        L.ref_decompress.restype = C.c_int

    def analyze(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.uint16)
        top = np.zeros(7, np.int32)
        self.lib.ref_analyze(_ptr(a), a.shape[0], a.shape[1], _ptr(top))
        return top

    def init_matrices(self, M: int, K: int, N: int, seed: int = 12345):
        A = np.zeros((M, K), np.uint16)
        B = np.zeros((N, K), np.uint16)
        self.lib.ref_init_matrices(_ptr(A), _ptr(B), M, K, N, seed)
        return A, B

    def encode(self, a: np.ndarray, top=None, variant: str = "reuse") -> Encoded:
        a = np.ascontiguousarray(a, np.uint16)
        M, K = a.shape
        if top is None:
            top = self.analyze(a)
        top = np.ascontiguousarray(top, np.int32)
        b = _alloc(M, K)
        s = np.zeros(4, np.int32)
        common = [_ptr(a), M, K, _ptr(top), _ptr(b["sm"]), _ptr(b["full"]), _ptr(b["b1"]),
                  _ptr(b["b2"]), _ptr(b["b3"]), _ptr(b["st"]), _ptr(b["mt"]), _ptr(b["gt"]),
                  _ptr(s[0:]), _ptr(s[1:])]
        if variant == "scalar":
            self.lib.ref_encode_scalar(*common)
        elif variant == "reuse":
            self.lib.ref_encode_reuse(*common, _ptr(s[2:]), _ptr(s[3:]))
        elif variant == "simd":
            self.lib.ref_encode_simd(*common, _ptr(s[2:]), _ptr(s[3:]))
        else:
            raise ValueError(variant)
        return _trim(b, s[0], s[1], top)


def have_reference() -> bool:
    return os.path.exists(REF_SO)
