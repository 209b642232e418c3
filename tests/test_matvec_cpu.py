"""The CPU restatement of the weight matvec (oracle/matvec.py) against the
reference: its committed golden outputs (tests/golden/matvec_kats.npz, from
the reference's own kernels) and, where the reference has been built here
(oracle/_ref), its kernels on more shapes."""
import os

import numpy as np
import pytest

from oracle import matvec as mv

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "matvec_kats.npz")


@pytest.mark.parametrize("name", sorted(mv.TYPES))
def test_restatement_matches_reference_goldens(name):
    g = np.load(GOLDEN)
    t = mv.TYPES[name]
    out_n, in_n = (int(v) for v in g[f"{name}_shape"])
    y = mv.matvec(t, g[f"{name}_W"], out_n, in_n, g[f"{name}_x"])
    ref = g[f"{name}_y"].astype(np.float64)
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref)), name


@pytest.mark.skipif(mv.ref_lib() is None, reason="oracle/_ref/libref_matvec.so not built")
@pytest.mark.parametrize("name", sorted(mv.TYPES))
@pytest.mark.parametrize("out_n,in_n", [(7, 256), (33, 4096)])
def test_restatement_matches_reference_kernels(name, out_n, in_n):
    t = mv.TYPES[name]
    rng = np.random.default_rng(out_n * 100 + t)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = rng.standard_normal(in_n, dtype=np.float32)
    ref = mv.ref_matvec(t, W, out_n, in_n, x).astype(np.float64)
    y = mv.matvec(t, W, out_n, in_n, x)[0]
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref)), name
