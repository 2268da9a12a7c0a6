"""C-ABI library: loads, exports every declared symbol, host encoder is
byte-identical to the reference fixtures (no GPU needed)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from golden_data import FIELDS, NAMES, load

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def zlib():
    from zipserv_asplos26_b200.build_lib import build
    build()
    from zipserv_asplos26_b200._lib import lib
    return lib()


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    return sorted(set(re.findall(r"\b(zs_[a-z0-9_]+)\s*\(", txt)))


def test_c_abi_exports_every_declared_symbol(zlib):
    for name in _declared("zipserv_b200.h"):
        assert hasattr(zlib, name), name


def test_cpp_abi_exports_reference_mangled_names(zlib):
    # build/L_API.cuh:19-165 names, C++-mangled exactly as the reference's.
    out = os.popen(f"nm -D --defined-only {zlib._name}").read()
    for name in ("BF16TripleBitmap_MM_API", "BF16TripleBitmap_Decompress_API", "InitBF16MatrixTripleBitmap",
                 "InitBF16MatrixTripleBitmap_Reuse", "InitBF16MatrixTripleBitmap_Reuse_SIMD",
                 "InitBF16MatrixTripleBitmap_GPU"):
        assert re.search(r"_Z\d+%sP" % name, out) or re.search(r"_Z\d+%s" % name, out), name
    # reference symbol spellings (from the reference's own object, recorded here)
    assert "_Z23BF16TripleBitmap_MM_APIP11CUstream_stPKhPK13__nv_bfloat16PKmS7_S7_PKiS9_iihS5_PS3_iiiSA_i" in out


def _encode_host(zlib, a, top):
    M, K = a.shape
    ngt = (M // 64) * (K // 64)
    nst = M * K // 64
    bufs = dict(sm=np.zeros(M * K + 16 * ngt, np.uint8), full=np.zeros(M * K + 8 * ngt, np.uint16),
                b1=np.zeros(nst, np.uint64), b2=np.zeros(nst, np.uint64), b3=np.zeros(nst, np.uint64),
                st=np.zeros(2 * nst, np.int32), mt=np.zeros(2 * nst // 16, np.int32),
                gt=np.zeros(2 * (ngt + 1), np.int32), sc=np.zeros(4, np.int32))
    p = lambda x: x.ctypes.data_as(C.c_void_p)  # noqa: E731
    a = np.ascontiguousarray(a)
    top = np.ascontiguousarray(top, np.int32)
    r = zlib.zs_encode_host(p(a), M, K, p(top), *(p(bufs[k]) for k in
                            ("sm", "full", "b1", "b2", "b3", "st", "mt", "gt", "sc")))
    assert r == 0
    return bufs


@pytest.mark.parametrize("name", NAMES)
def test_host_encoder_matches_reference_bytes(zlib, name):
    g = load(name)
    b = _encode_host(zlib, g["a"], g["top"])
    th, tf = b["gt"][-2], b["gt"][-1]
    assert np.array_equal(b["sm"][:th], g["sign_mantissa"])
    assert np.array_equal(b["full"][:tf], g["full"])
    for k, f in (("b1", "bitmap1"), ("b2", "bitmap2"), ("b3", "bitmap3"), ("st", "st_counts"),
                 ("mt", "mt_offsets"), ("gt", "gt_offsets")):
        assert np.array_equal(b[k], g[f]), f
    assert b["sc"][0] == g["max_hf"] and b["sc"][1] == g["max_full"]


@pytest.mark.parametrize("name", NAMES)
def test_host_window_rules(zlib, oracle, name):
    a = np.ascontiguousarray(load(name)["a"])
    for rule, rname in ((0, "host"), (1, "ext")):
        top = np.zeros(7, np.int32)
        assert zlib.zs_analyze_exponents_host(a.ctypes.data_as(C.c_void_p), a.size, rule,
                                              top.ctypes.data_as(C.c_void_p)) == 0
        assert np.array_equal(top, oracle.analyze(a, rname))


def test_invalid_shapes_rejected(zlib):
    a = np.zeros((64, 60), np.uint16)
    top = np.arange(120, 127, dtype=np.int32)
    z = np.zeros(8192, np.uint64)
    p = lambda x: x.ctypes.data_as(C.c_void_p)  # noqa: E731
    assert zlib.zs_encode_host(p(a), 64, 60, p(top), *([p(z)] * 9)) != 0


def test_compress_host_wrapper_matches_oracle(oracle):
    """The torch-facing host encoder returns the reference encoder's bytes."""
    import numpy as np
    import torch

    import zipserv_asplos26_b200 as zs
    rng = np.random.default_rng(3)
    w = torch.from_numpy(rng.standard_normal((128, 192), dtype=np.float32) * 0.02).to(torch.bfloat16)
    c = zs.compress_host(w)
    e = oracle.encode(w.view(torch.int16).numpy().view(np.uint16))
    assert c.start_exp == e.start_exp
    assert np.array_equal(c.sign_mantissa.numpy()[: e.total_hf], e.sign_mantissa[: e.total_hf])
    assert np.array_equal(c.compressed_full.view(torch.int16).numpy().view(np.uint16)[: e.total_full],
                          e.full[: e.total_full])
    for a, b in ((c.bitmap1, e.bitmap1), (c.bitmap2, e.bitmap2), (c.bitmap3, e.bitmap3)):
        assert np.array_equal(a.numpy().view(np.uint64), b)
    assert np.array_equal(c.tile_offsets_median.numpy(), e.mt_offsets)
    assert np.array_equal(c.tile_offsets_global.numpy(), e.gt_offsets)
