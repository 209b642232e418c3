"""The device matvec (pickle_cuda_matvec_dev) against the reference's own
outputs (tests/golden/matvec_kats.npz) and the CPU restatement
(oracle/matvec.py) at model sizes. Bar: 1e-4 relative to the largest
output, the FP32 bar of this library."""
import os

import numpy as np
import pytest
import torch

from oracle import matvec as mv
from lestramanika_b200 import PickleError, api

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "matvec_kats.npz")


def _run(t, W, out_n, in_n, x):
    x = np.atleast_2d(x)
    Wd = torch.from_numpy(np.ascontiguousarray(W)).to(DEV)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV)
    yd = torch.full((x.shape[0], out_n), float("nan"), device=DEV)
    api.matvec_dev(t, Wd, out_n, in_n, xd, yd, n_vec=x.shape[0])
    torch.cuda.synchronize()
    return yd.cpu().numpy().astype(np.float64)


def _close(got, ref, what):
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err <= 1e-4, (what, err)


@pytest.mark.parametrize("name", sorted(mv.TYPES))
def test_matvec_matches_reference_goldens(name):
    g = np.load(GOLDEN)
    out_n, in_n = (int(v) for v in g[f"{name}_shape"])
    got = _run(mv.TYPES[name], g[f"{name}_W"], out_n, in_n, g[f"{name}_x"])
    _close(got, g[f"{name}_y"].astype(np.float64), name)


@pytest.mark.parametrize("name", sorted(mv.TYPES))
@pytest.mark.parametrize("out_n,in_n,n_vec", [(1001, 4096, 1), (64, 14336, 3), (8, 256, 8), (5, 1024, 5),
                                              (33, 1536, 2), (70, 2048, 4), (17, 6144, 7)])
def test_matvec_matches_oracle_at_model_sizes(name, out_n, in_n, n_vec):
    t = mv.TYPES[name]
    rng = np.random.default_rng(out_n + in_n + t)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = rng.standard_normal((n_vec, in_n), dtype=np.float32)
    _close(_run(t, W, out_n, in_n, x), mv.matvec(t, W, out_n, in_n, x), f"{name} {out_n}x{in_n} n_vec={n_vec}")
    assert api.matvec_take_error(0) == 0


@pytest.mark.parametrize("name", ["F16", "Q4_0", "Q8_0"])
@pytest.mark.parametrize("out_n,in_n", [(3, 96), (40, 320)])
def test_matvec_rows_not_16_byte_multiples(name, out_n, in_n):
    # F16 rows of 96 or 320 halves, Q4_0 / Q8_0 rows of 3 or 10 blocks:
    # rows that do not start on 16-byte boundaries.
    t = mv.TYPES[name]
    rng = np.random.default_rng(in_n + t)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = rng.standard_normal((2, in_n), dtype=np.float32)
    _close(_run(t, W, out_n, in_n, x), mv.matvec(t, W, out_n, in_n, x), f"{name} {out_n}x{in_n}")


@pytest.mark.parametrize("name", sorted(mv.TYPES))
@pytest.mark.parametrize("scale", [1e-30, 1e-3, 1e3, 1e30])
def test_matvec_activation_magnitudes(name, scale):
    # The tensor-core path rescales x by a power of two per chunk before
    # splitting it into f16 halves; tiny and huge activations must come out
    # to the same relative accuracy. One chunk of x is all zeros.
    t = mv.TYPES[name]
    out_n, in_n = 48, 4096
    rng = np.random.default_rng(7 + t)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = (rng.standard_normal((2, in_n)) * scale).astype(np.float32)
    x[:, 1024:2048] = 0
    x[1, :512] *= 1e-6
    _close(_run(t, W, out_n, in_n, x), mv.matvec(t, W, out_n, in_n, x), f"{name} scale {scale}")


def test_matvec_errors():
    W = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    x = torch.zeros(256, device=DEV)
    y = torch.zeros(8, device=DEV)
    with pytest.raises(PickleError) as e:
        api.matvec_dev(3, W, 8, 256, x, y)               # Q4_1: not on the device path
    assert e.value.code == -4                            # PICKLE_ERR_TYPE, as the reference's dispatch
    with pytest.raises(PickleError) as e:
        api.matvec_dev(mv.TYPES["Q4_K"], W, 1, 128, x, y)   # not a whole Q4_K block
    assert e.value.code == -6
    with pytest.raises(PickleError) as e:
        api.matvec_dev(0, W, 1, 256, x, y, n_vec=9)
    assert e.value.code == -6
