"""Generate the golden TCA-TBE fixtures in this directory.

Each fixture is produced by the REFERENCE's own host code, compiled from its
sources into oracle/_ref/libzipserv_ref.so (`make -C oracle ref`):
  * exponent window  -- kernel_benchmark/utils.h:189 analyzeExponentDistribution_BF16
  * encoded streams  -- csrc/L_API.cu:559 InitBF16MatrixTripleBitmap_Reuse
                        (cross-checked here against csrc/L_API.cu:314 and :804,
                        which must agree byte for byte)
  * 'refgen' inputs  -- kernel_benchmark/utils.h:101 init_host_matrices_bf16 (seed 12345)
Other inputs are seeded numpy draws rounded to bf16 (round-to-nearest-even).

Run once in a container where the reference tree exists:
    make -C oracle all ref && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle_bindings import Reference  # noqa: E402


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def cases(ref: Reference):
    rng = np.random.default_rng(2024)
    a, b = ref.init_matrices(128, 192, 16, 12345)
    yield "refgen_128x192", a, b
    yield "normal002_256x256", f32_to_bf16_bits(rng.normal(0, 0.02, (256, 256))), None
    yield "normal1_64x320", f32_to_bf16_bits(rng.normal(0, 1.0, (64, 320))), None
    scale = np.exp(rng.uniform(np.log(0.1), np.log(4.0), 128))
    yield "kvlike_128x128", f32_to_bf16_bits(rng.normal(0, 1, (128, 128)) * scale[None, :]), None
    w = rng.normal(0, 1, (64, 64)) * np.exp(rng.uniform(-12, 12, (64, 64)))
    yield "wide_64x64", f32_to_bf16_bits(w), None
    sp = f32_to_bf16_bits(rng.normal(0, 0.05, (128, 128)))
    idx = rng.choice(sp.size, 600, replace=False)
    specials = np.array([0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x0001, 0x807F, 0x7F7F, 0x0080],
                        np.uint16)
    sp.reshape(-1)[idx] = specials[rng.integers(0, specials.size, idx.size)]
    yield "specials_128x128", sp, None
    yield "zeros_64x128", np.zeros((64, 128), np.uint16), None
    few = np.full((64, 64), 0x3F80, np.uint16)            # 1.0, exponent 127
    few[::3, :] = 0x4000                                  # 2.0, exponent 128
    few[:, ::5] = 0xBE00                                  # -0.125, exponent 124
    yield "fewexps_64x64", few, None
    exps = np.array([100, 102, 104, 106, 108, 110, 112, 114], np.uint16)
    e = exps[rng.integers(0, 8, (64, 128))]
    nc = (rng.integers(0, 2, (64, 128)).astype(np.uint16) << 15) | (e << 7) | rng.integers(0, 128, (64, 128)).astype(np.uint16)
    yield "noncontig_64x128", nc.astype(np.uint16), None
    pad = np.zeros((256, 128), np.uint16)                 # KV-style zero padding
    pad[:150] = f32_to_bf16_bits(rng.normal(0, 1, (150, 128)) * scale[None, :])
    yield "padded_256x128", pad, None


def main():
    ref = Reference()
    for name, a, b in cases(ref):
        top = ref.analyze(a)
        enc = ref.encode(a, top, "reuse")
        for v in ("scalar", "simd"):
            other = ref.encode(a, top, v)
            for f in ("sign_mantissa", "full", "bitmap1", "bitmap2", "bitmap3", "st_counts",
                      "mt_offsets", "gt_offsets"):
                assert np.array_equal(getattr(enc, f), getattr(other, f)), (name, v, f)
            assert (enc.max_hf, enc.max_full) == (other.max_hf, other.max_full), (name, v)
        out = dict(a=a, top=top, sign_mantissa=enc.sign_mantissa, full=enc.full,
                   bitmap1=enc.bitmap1, bitmap2=enc.bitmap2, bitmap3=enc.bitmap3,
                   st_counts=enc.st_counts, mt_offsets=enc.mt_offsets, gt_offsets=enc.gt_offsets,
                   max_hf=np.int32(enc.max_hf), max_full=np.int32(enc.max_full))
        if b is not None:
            out["b"] = b
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(f"{name}: top={top.tolist()} hf={enc.total_hf} full={enc.total_full} "
              f"max=({enc.max_hf},{enc.max_full})")


if __name__ == "__main__":
    main()
