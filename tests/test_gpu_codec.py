"""GPU parity: encoder bytes, decoder round trip, ZipGEMM numerics.

Checked against the CPU oracle (itself pinned to reference-built fixtures) and,
where available, the reference kernels compiled from source for sm_100a."""
import numpy as np
import pytest
import torch

from golden_data import FIELDS, NAMES, load

pytestmark = pytest.mark.gpu

# rel-L2 against the exact product rounded to bf16 -- what any fp32-accumulate,
# bf16-output GEMM (the reference's included) produces up to summation order.
GEMM_TOL = 1e-3


@pytest.fixture(scope="module")
def zs():
    import zipserv_asplos26_b200 as z
    from zipserv_asplos26_b200._lib import lib
    lib()
    return z


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def gen_w(M, K, seed, sigma=0.02):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(M, K, generator=g, device="cuda") * sigma).to(torch.bfloat16)


@pytest.mark.parametrize("name", NAMES)
def test_gpu_encoder_bytes_match_reference(zs, name):
    g = load(name)
    c = zs.compress(to_dev(g["a"]), top=torch.from_numpy(g["top"]))
    torch.cuda.synchronize()
    assert np.array_equal(c.sign_mantissa[: c.total_hf].cpu().numpy(), g["sign_mantissa"])
    assert np.array_equal(bits(c.compressed_full[: c.total_full]), g["full"])
    for ours, f in ((c.bitmap1, "bitmap1"), (c.bitmap2, "bitmap2"), (c.bitmap3, "bitmap3")):
        assert np.array_equal(ours.cpu().view(torch.int64).numpy().view(np.uint64), g[f]), f
    assert np.array_equal(c.tile_offsets.cpu().numpy(), g["st_counts"])
    assert np.array_equal(c.tile_offsets_median.cpu().numpy(), g["mt_offsets"])
    assert np.array_equal(c.tile_offsets_global.cpu().numpy(), g["gt_offsets"])
    assert (c.max_high_freq_count, c.max_full_count) == (int(g["max_hf"]), int(g["max_full"]))


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("rule", ["host", "ext"])
def test_gpu_window_rules(zs, oracle, name, rule):
    a = load(name)["a"]
    top = zs.analyze_exponents(to_dev(a), rule).cpu().numpy()
    assert np.array_equal(top, oracle.analyze(a, rule))


@pytest.mark.parametrize("name", NAMES)
def test_gpu_decompress_round_trip_golden(zs, name):
    g = load(name)
    c = zs.compress(to_dev(g["a"]), top=torch.from_numpy(g["top"]))
    out = zs.decompress(c)
    assert np.array_equal(bits(out), g["a"])


@pytest.mark.parametrize("shape,seed", [((1024, 2048), 1), ((192, 4096), 2), ((4096, 4096), 3)])
def test_gpu_round_trip_large(zs, oracle, shape, seed):
    w = gen_w(*shape, seed)
    c = zs.compress(w)
    out = zs.decompress(c)
    assert torch.equal(out.view(torch.int16), w.view(torch.int16))
    # same bytes as the CPU oracle encoder
    e = oracle.encode(bits(w), np.array(c.top, np.int32))
    assert np.array_equal(c.sign_mantissa[: c.total_hf].cpu().numpy(), e.sign_mantissa)
    assert np.array_equal(c.tile_offsets_global.cpu().numpy(), e.gt_offsets)


def test_gpu_round_trip_kv_like_and_specials(zs):
    g = torch.Generator(device="cuda").manual_seed(7)
    scale = torch.exp(torch.empty(128, device="cuda").uniform_(np.log(0.1), np.log(4.0), generator=g))
    w = (torch.randn(2048, 128, generator=g, device="cuda") * scale).to(torch.bfloat16)
    w.view(torch.int16)[::37, ::5] = 0x7F80  # +inf
    w.view(torch.int16)[::41, ::7] = 0x7FC1  # NaN payload
    w.view(torch.int16)[::13, ::3] = 0       # zeros
    for rule in ("host", "ext"):
        c = zs.compress(w, rule)
        assert torch.equal(zs.decompress(c).view(torch.int16), w.view(torch.int16))


def test_gpu_all_fallback_tiles(zs):
    w = torch.zeros(256, 256, dtype=torch.bfloat16, device="cuda")
    c = zs.compress(w)
    assert c.total_hf == 0
    assert torch.equal(zs.decompress(c).view(torch.int16), w.view(torch.int16))


def _gemm_check(zs, oracle, M, K, N, seed, split_k=1, use_oracle=False):
    w = gen_w(M, K, seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 100)
    x = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
    c = zs.compress(w)
    y = zs.zipgemm(c, x, split_k=split_k)
    torch.cuda.synchronize()
    if use_oracle:
        ref = oracle.gemm(bits(w), bits(x))
    else:
        ref = (x.double() @ w.double().t()).cpu().numpy()
    ref_bf16 = torch.from_numpy(np.asarray(ref)).to(torch.bfloat16).double().numpy()
    err = rel_l2(y.double().cpu().numpy(), ref_bf16)
    assert err <= GEMM_TOL, (M, K, N, err)
    return err


@pytest.mark.parametrize("M,K,N", [(128, 192, 16), (64, 64, 1), (192, 128, 7), (128, 256, 40)])
def test_gpu_zipgemm_vs_oracle(zs, oracle, M, K, N):
    _gemm_check(zs, oracle, M, K, N, seed=11, use_oracle=True)


@pytest.mark.parametrize("N", [1, 8, 16, 17, 64, 100, 128, 256, 300])
def test_gpu_zipgemm_config2_shapes(zs, oracle, N):
    _gemm_check(zs, oracle, 4096, 4096, N, seed=N)


@pytest.mark.parametrize("M,K", [(6144, 4096), (4096, 14336), (1280, 8192), (576, 1024)])
def test_gpu_zipgemm_llama_shapes(zs, oracle, M, K):
    _gemm_check(zs, oracle, M, K, 32, seed=M + K)


@pytest.mark.parametrize("split_k", [1, 2, 4, 8])
def test_gpu_zipgemm_split_k_consistent(zs, oracle, split_k):
    _gemm_check(zs, oracle, 1024, 4096, 64, seed=5, split_k=split_k)


def test_gpu_zipgemm_vs_reference_kernel(zs):
    """Same inputs through the reference BF16TripleBitmap_MM_API (compiled from
    its sources for sm_100a): outputs agree within the GEMM tolerance."""
    from oracle_bindings import REF_SO, Reference, have_reference
    if not have_reference():
        pytest.skip("oracle/_ref not built")
    import ctypes as C
    ref = Reference(REF_SO)
    M = K = 4096
    N = 128
    w = gen_w(M, K, 0)
    x = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    c = zs.compress(w)
    ours = zs.zipgemm(c, x)
    # the reference kernel prefetches offsets two tiles past the array end (L_Kernel.cuh:444-447)
    gt_pad = torch.cat([c.tile_offsets_global, torch.zeros(16, dtype=torch.int32, device="cuda")])
    out_ref = torch.empty(N, M, dtype=torch.bfloat16, device="cuda")
    st = ref.lib.ref_mm(C.c_void_p(torch.cuda.current_stream().cuda_stream), c.sign_mantissa.data_ptr(),
                        c.compressed_full.data_ptr(), c.bitmap1.data_ptr(), c.bitmap2.data_ptr(),
                        c.bitmap3.data_ptr(), c.tile_offsets_median.data_ptr(), gt_pad.data_ptr(),
                        c.max_high_freq_count, c.max_full_count, c.start_exp, x.data_ptr(), out_ref.data_ptr(),
                        M, N, K, None, 1)
    assert st == 0
    torch.cuda.synchronize()
    exact = (x.double() @ w.double().t()).to(torch.bfloat16).double()
    assert rel_l2(ours.double().cpu(), exact.cpu()) <= GEMM_TOL
    assert rel_l2(out_ref.double().cpu(), exact.cpu()) <= GEMM_TOL
    assert rel_l2(ours.double().cpu(), out_ref.double().cpu()) <= GEMM_TOL


@pytest.mark.parametrize("M,K,N", [(128000, 64, 32), (16384, 256, 256), (64, 8192, 16), (8192, 1024, 200)])
def test_gpu_zipgemm_stream_k_segments(zs, oracle, M, K, N):
    """Shapes whose stream-K ranges cover many output tiles per CTA (drains
    during the run), a single 64-row tile split over every SM, and N > 128."""
    _gemm_check(zs, oracle, M, K, N, seed=M + N)


@pytest.mark.parametrize("mode", ["1", "0"])
@pytest.mark.parametrize("M,K,N", [(4096, 4096, 128), (28672, 4096, 16), (57344, 1024, 300), (8256, 192, 7),
                                   (20032, 320, 40)])
def test_gpu_zipgemm_persistent_mode(zs, oracle, monkeypatch, mode, M, K, N):
    """Persistent launch (one CTA per SM looping over tiles, two TMEM
    accumulators, epilogue warps) forced on (1) and off (0): several tiles per
    CTA, a half tile (M % 128 = 64) among them, odd K-block counts (one-unit
    chunks), N > 256 (two column chunks)."""
    monkeypatch.setenv("ZS_ZIPGEMM_PERSIST", mode)
    _gemm_check(zs, oracle, M, K, N, seed=M + K + N)


def test_gpu_zipgemm_deterministic(zs):
    """The split-tile reduction sums partials in a fixed order: repeated runs
    are bit-identical."""
    w = gen_w(4096, 4096, 3)
    x = torch.randn(128, 4096, device="cuda").to(torch.bfloat16)
    c = zs.compress(w)
    y0 = zs.zipgemm(c, x)
    for _ in range(5):
        assert torch.equal(zs.zipgemm(c, x).view(torch.int16), y0.view(torch.int16))


@pytest.mark.parametrize("counts", [[512] * 8, [455] * 8 + [456], [300, 700, 700, 300, 300, 700, 300, 300, 496],
                                    [1] * 3 + [1000] * 2 + [1] * 6 + [2087]])
@pytest.mark.parametrize("rule", ["host", "ext"])
def test_gpu_window_rules_with_ties(zs, oracle, counts, rule):
    """Histograms with equal counts at the seventh place, where the two rules'
    tie-breaking (arg-max passes vs a replace-the-minimum slot list) decides
    the window: the GPU picks what the reference-restating oracle picks."""
    rng = np.random.default_rng(len(counts) + sum(counts))
    exps = np.repeat(np.arange(100, 100 + len(counts)), counts)
    rng.shuffle(exps)
    a = ((exps.astype(np.uint16) << 7) | rng.integers(0, 128, exps.size).astype(np.uint16)).reshape(64, 64)
    top = zs.analyze_exponents(to_dev(a), rule).cpu().numpy()
    assert np.array_equal(top, oracle.analyze(a, rule))
