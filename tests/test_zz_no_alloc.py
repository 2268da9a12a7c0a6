"""The allocation-free decode-attention entry point (zs_decode_attention_noalloc).

It exists for callers that cannot allocate device memory while they run
attention (for example code running inside an allocator's own hooks, or a
deployment that forbids cudaMalloc after start-up to keep its memory budget
fixed): its split-KV workspace is a fixed array inside the library. This test
calls it through the C ABI, twice in a row, and checks each result against the
regular entry point (caller-provided workspace) within the attention tolerance.
It lives in its own file, collected last, so a failure here leaves every other
test already run."""
import ctypes as C
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-3  # rel-L2, same tolerance as the other attention tests

FIELDS = ("sign_mantissa", "compressed_full", "bitmap1", "bitmap2", "bitmap3", "tile_offsets_median",
          "tile_offsets_global")


def _args(c):
    ptrs = (C.c_void_p * 7)(*[getattr(c, f).data_ptr() for f in FIELDS])
    meta = (C.c_int * 5)(c.rows, c.cols, c.max_high_freq_count, c.max_full_count, c.start_exp)
    return ptrs, meta


def _kv(B, T, Hkv, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = torch.exp(torch.empty(D, device="cuda").uniform_(math.log(0.1), math.log(4.0), generator=g))
    return (torch.randn(B, T, Hkv, D, generator=g, device="cuda") * s).to(torch.bfloat16)


def _lib():
    from zipserv_asplos26_b200._lib import lib
    L = lib()
    L.zs_decode_attention_noalloc.argtypes = ([C.c_void_p] * 7 + [C.c_int] * 6 +
                                              [C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p])
    L.zs_decode_attention_noalloc.restype = C.c_int
    L.zs_decode_attention_noalloc_max_workspace_bytes.argtypes = []
    L.zs_decode_attention_noalloc_max_workspace_bytes.restype = C.c_size_t
    return L


def test_noalloc_attention_matches_regular_entry_point_twice():
    import zipserv_asplos26_b200 as zs
    L = _lib()

    B, T, Hq, Hkv, D, splits = 3, 1000, 32, 8, 128, 8
    t_pad = (T + 63) // 64 * 64
    kc = zs.compress_kv(_kv(B, T, Hkv, D, 1))
    vc = zs.compress_kv(_kv(B, T, Hkv, D, 2))
    kp, km = _args(kc)
    vp, vm = _args(vc)
    lens = torch.tensor([T, 700, 5], dtype=torch.int32, device="cuda")
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream

    # regular entry point with a caller-allocated workspace
    ws_bytes = L.zs_decode_attention_workspace_bytes(B, Hq, Hkv, splits)
    assert 0 < ws_bytes <= L.zs_decode_attention_noalloc_max_workspace_bytes()
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    for call in range(2):
        q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 + call))
        q = q.to(torch.bfloat16)
        ref = torch.empty_like(q)
        out = torch.full_like(q, float("nan"))
        used = C.c_int(0)
        assert L.zs_decode_attention(stream, q.data_ptr(), kp, km, vp, vm, lens.data_ptr(), B, Hq, Hkv, D, t_pad,
                                     T, scale, splits, ws.data_ptr(), ws_bytes, ref.data_ptr(), None, None) == 0
        assert L.zs_decode_attention_noalloc(stream, q.data_ptr(), kp, km, vp, vm, lens.data_ptr(), B, Hq, Hkv,
                                             D, t_pad, T, scale, splits, out.data_ptr(), C.byref(used), None) == 0
        torch.cuda.synchronize()
        assert used.value == splits
        err = float((out.double() - ref.double()).norm() / ref.double().norm())
        assert err <= TOL, (call, err)


def test_noalloc_attention_rejects_workspace_beyond_its_array():
    """A shape whose split-KV workspace exceeds the fixed array is refused with
    an error status. Every input is real and valid for that shape (B=8, 8 query
    and 8 KV heads, T=4096, 64 splits: 2.13 MB of workspace against the 2 MiB
    array), so if the size check ever regressed the call would compute into
    real buffers instead of touching unmapped addresses."""
    import zipserv_asplos26_b200 as zs
    L = _lib()
    cap = L.zs_decode_attention_noalloc_max_workspace_bytes()
    B, T, Hq, Hkv, D, splits = 8, 4096, 8, 8, 128, 64
    assert L.zs_decode_attention_workspace_bytes(B, Hq, Hkv, splits) > cap
    kc = zs.compress_kv(_kv(B, T, Hkv, D, 3))
    vc = zs.compress_kv(_kv(B, T, Hkv, D, 4))
    kp, km = _args(kc)
    vp, vm = _args(vc)
    q = torch.randn(B, Hq, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)).to(torch.bfloat16)
    lens = torch.full((B,), T, dtype=torch.int32, device="cuda")
    out = torch.full_like(q, 7.0)
    used = C.c_int(-1)
    rc = L.zs_decode_attention_noalloc(torch.cuda.current_stream().cuda_stream, q.data_ptr(), kp, km, vp, vm,
                                       lens.data_ptr(), B, Hq, Hkv, D, T, T, 1.0 / math.sqrt(D), splits,
                                       out.data_ptr(), C.byref(used), None)
    torch.cuda.synchronize()
    assert rc != 0
    assert used.value == -1                      # nothing was launched
    assert bool((out == 7.0).all())              # the output was not written
