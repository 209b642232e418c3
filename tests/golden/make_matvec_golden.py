"""Generate tests/golden/matvec_kats.npz: for each weight format the device
matvec takes, seeded random raw weights W, activations x and the
reference's own output y, from its kernels compiled from its sources
(oracle/_ref/libref_matvec.so, built by `make -C oracle ref`).

    python tests/golden/make_matvec_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import matvec as mv  # noqa: E402

SHAPES = {"F32": (24, 256), "F16": (24, 512), "Q4_0": (40, 512), "Q8_0": (40, 512), "Q4_K": (40, 768),
          "Q6_K": (40, 768)}


def main():
    if mv.ref_lib() is None:
        sys.exit("oracle/_ref/libref_matvec.so is not built")
    out = {}
    for name, t in mv.TYPES.items():
        rng = np.random.default_rng(1000 + t)
        out_n, in_n = SHAPES[name]
        W = mv.random_weights(t, out_n, in_n, rng)
        x = rng.standard_normal((2, in_n), dtype=np.float32)
        y = np.stack([mv.ref_matvec(t, W, out_n, in_n, x[v]) for v in range(2)])
        out[f"{name}_W"] = W
        out[f"{name}_x"] = x
        out[f"{name}_y"] = y
        out[f"{name}_shape"] = np.array([out_n, in_n], np.int32)
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "matvec_kats.npz"), **out)


if __name__ == "__main__":
    main()
