"""On-disk TCA-TBE container (zs_tcatbe_save / read_info / load through the C
ABI): exact round trip of every array, checksum and format rejection, and a
loaded file feeding the GPU decoder and ZipGEMM."""
import numpy as np
import pytest
import torch

import zipserv_asplos26_b200 as zs
from zipserv_asplos26_b200 import store
from zipserv_asplos26_b200._lib import ZipServError


def _weight(M, K, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32) * scale).to(torch.bfloat16)


def _bits(t, n=None):
    t = t.reshape(-1) if n is None else t.reshape(-1)[:n]
    dt = {torch.bfloat16: torch.int16, torch.uint64: torch.int64}.get(t.dtype, t.dtype)
    return t.cpu().view(dt).numpy().copy()


def _assert_same(a, b, with_st=True):
    assert (a.rows, a.cols, a.start_exp, a.max_high_freq_count, a.max_full_count, a.total_hf, a.total_full) == \
           (b.rows, b.cols, b.start_exp, b.max_high_freq_count, b.max_full_count, b.total_hf, b.total_full)
    assert list(a.top) == list(b.top)
    assert np.array_equal(_bits(a.sign_mantissa, a.total_hf), _bits(b.sign_mantissa, b.total_hf))
    assert np.array_equal(_bits(a.compressed_full, a.total_full), _bits(b.compressed_full, b.total_full))
    for x, y in ((a.bitmap1, b.bitmap1), (a.bitmap2, b.bitmap2), (a.bitmap3, b.bitmap3),
                 (a.tile_offsets_median, b.tile_offsets_median), (a.tile_offsets_global, b.tile_offsets_global)):
        assert np.array_equal(_bits(x), _bits(y))
    if with_st:
        assert np.array_equal(_bits(a.tile_offsets), _bits(b.tile_offsets))


@pytest.mark.parametrize("shape,seed,scale", [((128, 192), 1, 0.02), ((64, 64), 2, 1.0), ((192, 128), 3, 30.0)])
def test_save_load_round_trip_is_exact(tmp_path, oracle, shape, seed, scale):
    w = _weight(*shape, seed, scale)
    c = zs.compress_host(w)
    path = tmp_path / "w.zst"
    store.save(c, path)
    info = store.read_info(path)
    assert (info["rows"], info["cols"], info["total_hf"], info["total_full"]) == (*shape, c.total_hf, c.total_full)
    assert info["has_st_counts"]
    d = store.load(path, with_st_counts=True)
    _assert_same(c, d)
    # the loaded arrays decode back to the original matrix (oracle decoder)
    from oracle_bindings import Encoded
    e = Encoded(_bits(d.sign_mantissa, d.total_hf).view(np.uint8), _bits(d.compressed_full, d.total_full).view(np.uint16),
                _bits(d.bitmap1).view(np.uint64), _bits(d.bitmap2).view(np.uint64), _bits(d.bitmap3).view(np.uint64),
                _bits(d.tile_offsets), _bits(d.tile_offsets_median), _bits(d.tile_offsets_global),
                d.max_high_freq_count, d.max_full_count, np.asarray(d.top, np.int32))
    out = oracle.decode(e, *shape, start_exp=d.start_exp)
    assert np.array_equal(out, w.view(torch.int16).numpy().view(np.uint16))


def test_load_without_small_tile_counts(tmp_path):
    c = zs.compress_host(_weight(64, 128, 4))
    c.tile_offsets = None
    path = tmp_path / "w.zst"
    store.save(c, path)
    assert not store.read_info(path)["has_st_counts"]
    d = store.load(path, with_st_counts=True)
    assert d.tile_offsets is None
    _assert_same(c, d, with_st=False)


def test_damaged_foreign_and_missing_files_are_rejected(tmp_path):
    c = zs.compress_host(_weight(128, 128, 5))
    path = tmp_path / "w.zst"
    store.save(c, path)
    raw = bytearray(path.read_bytes())
    # a flipped byte in the sign/mantissa stream fails its checksum
    bad = bytearray(raw)
    bad[512 + 7] ^= 0x40
    (tmp_path / "flip.zst").write_bytes(bytes(bad))
    with pytest.raises(ZipServError, match="status 1"):
        store.load(tmp_path / "flip.zst")
    # a truncated file is a short read
    (tmp_path / "short.zst").write_bytes(bytes(raw[: len(raw) - 100]))
    with pytest.raises(ZipServError, match="status 999"):
        store.load(tmp_path / "short.zst")
    # another format, or a different version, is refused at the header
    (tmp_path / "foreign.bin").write_bytes(b"NOTAFILE" + bytes(raw[8:]))
    with pytest.raises(ZipServError, match="status 1"):
        store.read_info(tmp_path / "foreign.bin")
    ver = bytearray(raw)
    ver[8] = 2
    (tmp_path / "v2.zst").write_bytes(bytes(ver))
    with pytest.raises(ZipServError, match="status 1"):
        store.load(tmp_path / "v2.zst")
    with pytest.raises(ZipServError, match="status 301"):
        store.read_info(tmp_path / "missing.zst")


def test_save_rejects_inconsistent_sizes(tmp_path):
    c = zs.compress_host(_weight(64, 64, 6))
    c.rows = 100    # not a multiple of 64
    with pytest.raises(ZipServError, match="status 1"):
        store.save(c, tmp_path / "x.zst")


@pytest.mark.gpu
def test_loaded_file_feeds_gpu_decoder_and_zipgemm(tmp_path):
    """A file written from a GPU-compressed matrix loads onto the GPU and gives
    the same decompressed matrix and the same ZipGEMM output, bit for bit."""
    torch.manual_seed(7)
    w = (torch.randn(256, 512, device="cuda") * 0.02).to(torch.bfloat16)
    c = zs.compress(w)
    path = tmp_path / "w.zst"
    store.save(c, path)
    d = store.load(path, device="cuda")
    assert torch.equal(zs.decompress(d).view(torch.int16), w.view(torch.int16))
    x = torch.randn(64, 512, device="cuda").to(torch.bfloat16)
    assert torch.equal(zs.zipgemm(d, x).view(torch.int16), zs.zipgemm(c, x).view(torch.int16))


@pytest.mark.parametrize("how", ["tile_too_long", "decreasing", "median_outside_tile", "median_nonzero_start"])
def test_load_rejects_offsets_that_do_not_describe_the_streams(tmp_path, how):
    """A file whose checksums are consistent but whose offsets are not (a buggy
    writer, or a crafted file) is refused on load: decoders would otherwise be
    sent past the staged streams."""
    c = zs.compress_host(_weight(128, 128, 7))
    gt = c.tile_offsets_global.clone()
    mt = c.tile_offsets_median.clone()
    if how == "tile_too_long":      # tile 0 claims tile 1's hf bytes too: more than max_hf allows
        gt[2] = gt[4]
    elif how == "decreasing":       # the fallback offsets of tile 1 go backwards
        gt[3] = gt[5] + 8
    elif how == "median_outside_tile":
        mt[2] = int(gt[2]) + 16     # median tile 1 of tile 0 starts past the tile's end
    else:
        mt[0] = 16
    c.tile_offsets_global, c.tile_offsets_median = gt, mt
    path = tmp_path / "bad.zst"
    store.save(c, path)             # the writer checksums whatever it is given
    with pytest.raises(ZipServError):
        store.load(path)
