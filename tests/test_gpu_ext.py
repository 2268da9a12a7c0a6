"""The reference extension's surface (compress_zipserv / decompress_zipserv[_into])."""
import numpy as np
import pytest
import torch

from golden_data import load

pytestmark = pytest.mark.gpu


def test_compress_zipserv_outputs_and_meta(oracle):
    from zipserv_asplos26_b200 import ext
    g = load("kvlike_128x128")
    a = torch.from_numpy(g["a"].view(np.int16)).view(torch.bfloat16).cuda()
    outs = ext.compress_zipserv(a, 100, 120)
    assert len(outs) == 8
    sm, full, b1, b2, b3, mt, gt, meta = outs
    m = meta.tolist()
    top = oracle.analyze(g["a"], "ext")
    e = oracle.encode(g["a"], top)
    assert m[:4] == [128, 128, 100, 120]
    assert m[4:10] == [e.max_hf, e.max_full, int(top[0]) - 1, e.total_hf, e.total_full, 4]
    assert m[10] == e.compressed_bytes() + 8 * b1.numel() + 28
    assert sm.numel() == 128 * 128 and full.numel() == 128 * 128
    assert np.array_equal(sm[: e.total_hf].cpu().numpy(), e.sign_mantissa)
    assert np.array_equal(gt.cpu().numpy(), e.gt_offsets)
    dense = ext.decompress_zipserv(sm, full, b1, b2, b3, mt, gt, 128, 128, m[4], m[5], m[6])
    assert torch.equal(dense.view(torch.int16), a.view(torch.int16))
    out = torch.empty_like(a)
    ext.decompress_zipserv_into(out, sm, full, b1, b2, b3, mt, gt, 128, 128, m[4], m[5], m[6])
    assert torch.equal(out.view(torch.int16), a.view(torch.int16))


def test_ext_input_checks():
    from zipserv_asplos26_b200 import ext
    with pytest.raises(RuntimeError, match="bfloat16"):
        ext.compress_zipserv(torch.zeros(64, 64, device="cuda"), 64, 64)
    with pytest.raises(RuntimeError, match="multiple of 64"):
        ext.compress_zipserv(torch.zeros(64, 96, device="cuda", dtype=torch.bfloat16), 64, 96)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.compress_zipserv(torch.zeros(64, 64, dtype=torch.bfloat16), 64, 64)
