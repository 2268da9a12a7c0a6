"""Loader for the committed golden fixtures (tests/golden/*.npz)."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
FIELDS = ("sign_mantissa", "full", "bitmap1", "bitmap2", "bitmap3", "st_counts", "mt_offsets",
          "gt_offsets")


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, name + ".npz")) as z:
        return {k: z[k] for k in z.files}
