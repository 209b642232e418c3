"""The batched matmul (pickle_cuda_matmul_dev: the reference's per-token
pickle_fast_matmul_dispatch over a whole prompt) against the CPU
restatement (oracle/matvec.py, float64 dot products of the reference's
dequantized weights). Bar: 1e-4 relative to the largest output, as the
matvec. F16, Q8_0, Q4_0, Q4_K and Q6_K with a workspace, 16-byte multiple
rows and in_n a multiple of 256 take the tensor-core GEMM; the other cases
run the matvec in passes and are checked the same way."""
import numpy as np
import pytest
import torch

from oracle import matvec as mv
from lestramanika_b200 import PickleError, api

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _run(t, W, out_n, in_n, x, use_ws=True):
    n_tok = x.shape[0]
    Wd = torch.from_numpy(np.ascontiguousarray(W)).to(DEV)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV)
    yd = torch.full((n_tok, out_n), float("nan"), device=DEV)
    ws = None
    if use_ws:
        ws = torch.empty(api.matmul_workspace(out_n, in_n, n_tok), dtype=torch.uint8, device=DEV)
    api.matmul_dev(t, Wd, out_n, in_n, xd, yd, n_tok, workspace=ws)
    torch.cuda.synchronize()
    assert api.matvec_take_error(0) == 0
    return yd.cpu().numpy().astype(np.float64)


def _close(got, ref, what):
    err = np.max(np.abs(got - ref)) / np.max(np.abs(ref))
    assert err <= 1e-4, (what, err)


@pytest.mark.parametrize("name", ["Q4_K", "F16", "Q8_0", "Q4_0", "Q6_K"])
@pytest.mark.parametrize("out_n,in_n,n_tok", [(256, 4096, 64), (300, 512, 200), (128, 1024, 9), (70, 256, 257),
                                              (130, 2048, 40)])
def test_matmul_tensor_core_path(name, out_n, in_n, n_tok):
    t = mv.TYPES[name]
    rng = np.random.default_rng(out_n * 7 + in_n + n_tok + t)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = rng.standard_normal((n_tok, in_n), dtype=np.float32)
    _close(_run(t, W, out_n, in_n, x), mv.matvec(t, W, out_n, in_n, x), f"{name} {out_n}x{in_n} T={n_tok}")


@pytest.mark.parametrize("name", sorted(mv.TYPES))
def test_matmul_every_type_with_and_without_workspace(name):
    # F32, rows that are not 16-byte multiples (Q6_K at in_n 512) and calls
    # without a workspace run the matvec in passes of eight rows.
    t = mv.TYPES[name]
    out_n, in_n, n_tok = 96, 512, 21
    rng = np.random.default_rng(t + 99)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = rng.standard_normal((n_tok, in_n), dtype=np.float32)
    ref = mv.matvec(t, W, out_n, in_n, x)
    _close(_run(t, W, out_n, in_n, x), ref, name)
    _close(_run(t, W, out_n, in_n, x, use_ws=False), ref, name + " no workspace")


@pytest.mark.parametrize("name", ["Q4_K", "F16", "Q8_0", "Q6_K"])
@pytest.mark.parametrize("scale", [1e-20, 1e20])
def test_matmul_activation_magnitudes(name, scale):
    # Per-token power-of-two scaling before the f16 split; one token all zero.
    t = mv.TYPES[name]
    out_n, in_n, n_tok = 128, 2048, 24
    rng = np.random.default_rng(t + 5)
    W = mv.random_weights(t, out_n, in_n, rng)
    x = (rng.standard_normal((n_tok, in_n)) * scale).astype(np.float32)
    x[3] = 0
    got, ref = _run(t, W, out_n, in_n, x), mv.matvec(t, W, out_n, in_n, x)
    assert np.all(got[3] == 0)
    keep = np.arange(n_tok) != 3
    _close(got[keep], ref[keep], f"{name} scale {scale}")


def test_matmul_errors():
    W = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    x = torch.zeros((16, 256), device=DEV)
    y = torch.zeros((16, 8), device=DEV)
    with pytest.raises(PickleError) as e:
        api.matmul_dev(3, W, 8, 256, x, y, 16)            # Q4_1: not on the device path
    assert e.value.code == -4
    with pytest.raises(PickleError) as e:
        api.matmul_dev(mv.TYPES["Q4_K"], W, 8, 128, x, y, 16)   # not a whole Q4_K block
    assert e.value.code == -6
