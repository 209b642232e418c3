"""The device sampler (pickle_cuda_sample_dev) against the reference's own
pickle_fast_sample_temp (src/pickle_fast.c:2204-2276, called from
oracle/_ref/libref_matvec.so, the unmodified reference objects), and the
sampled decode loop (pickle_cuda_generate_sampled) against step-by-step
forward + sample calls.

The device sums probabilities as fixed-order trees where the reference keeps
one running float sum, so the two may pick neighbouring ids when the draw
lies within float rounding of a cumulative-probability boundary. The
parity test replays each case in float64 on the host and compares the ids
whenever every boundary the decision depends on is more than 1e-5 away;
at least 60 % of the cases must be compared, and every compared case must
match.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from lestramanika_b200 import api
from lestramanika_b200.model import PickleModel

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libref_matvec.so")
MARGIN = 1e-5


def _ref_sampler():
    if not os.path.exists(REF_LIB):
        pytest.fail(f"{REF_LIB} is not built (python -m lestramanika_b200.build --all)")
    f = ctypes.CDLL(REF_LIB).pickle_fast_sample_temp
    f.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
    f.restype = ctypes.c_int32
    return f


def _draw(seed):
    """One xorshift32 step from the seed, as the reference's sampler draws r."""
    x = seed if seed else 0x12345678
    x ^= (x << 13) & 0xFFFFFFFF
    x ^= x >> 17
    x ^= (x << 5) & 0xFFFFFFFF
    return float(np.float32(np.float32(x & 0xFFFFFF) / np.float32(0xFFFFFF)))


def _clear_of_boundaries(logits, temp, top_p, seed):
    """True when, in float64, no decision of the sampler is within MARGIN of a tie."""
    l = logits.astype(np.float64) / temp
    e = np.exp(l - l.max())
    p = e / e.sum()
    r = _draw(seed)
    if 0.0 < top_p < 1.0:
        order = np.argsort(-p, kind="stable")
        cum = np.cumsum(p[order])
        k = int(np.searchsorted(cum, top_p))              # first cum >= top_p
        k = min(k, len(cum) - 1)
        if abs(cum[k] - top_p) < MARGIN or (k > 0 and abs(cum[k - 1] - top_p) < MARGIN):
            return False
        R = r * cum[k]
        j = int(np.searchsorted(cum[:k + 1], R))
        j = min(j, k)
        return abs(cum[j] - R) >= MARGIN and (j == 0 or abs(cum[j - 1] - R) >= MARGIN)
    cum = np.cumsum(p)
    j = min(int(np.searchsorted(cum, r)), len(cum) - 1)
    return abs(cum[j] - r) >= MARGIN and (j == 0 or abs(cum[j - 1] - r) >= MARGIN)


@pytest.mark.parametrize("n,scale", [(32000, 3.0), (128256, 4.0), (4096, 0.3)])
def test_sampler_matches_reference(n, scale):
    ref = _ref_sampler()
    rng = np.random.default_rng(n)
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    compared = skipped = 0
    for case in range(60):
        x = (rng.standard_normal(n) * scale).astype(np.float32)
        temp = float(rng.choice([0.5, 0.8, 1.0, 1.3]))
        top_p = float(rng.choice([0.0, 0.5, 0.9, 0.95, 1.0]))
        seed = int(rng.integers(0, 2 ** 32))
        xr = x.copy()
        want = ref(xr.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n, temp, top_p, seed)
        xd = torch.from_numpy(x).to(DEV)
        api.sample_dev(xd, out, temp, top_p, seed)
        torch.cuda.synchronize()
        got = int(out.item())
        # both leave the logits as expf(logits / temp - max)
        np.testing.assert_allclose(xd.cpu().numpy(), xr, rtol=1e-5, atol=1e-30)
        if _clear_of_boundaries(x, temp, top_p, seed):
            assert got == want, (case, temp, top_p, seed, got, want)
            compared += 1
        else:
            skipped += 1
    # Nuclei of thousands of ids put neighbouring boundaries ~1e-5 apart, as
    # close as the reference's own float rounding: those cases are left out.
    assert compared >= 36, (compared, skipped)


def test_sampler_temp_zero_is_argmax():
    ref = _ref_sampler()
    x = np.random.default_rng(1).standard_normal(50000).astype(np.float32)
    x[[7, 4000]] = 9.0
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    xd = torch.from_numpy(x).to(DEV)
    api.sample_dev(xd, out, 0.0, 0.9, 5)
    torch.cuda.synchronize()
    xr = x.copy()
    assert int(out.item()) == ref(xr.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), x.size, 0.0, 0.9, 5) == 7
    np.testing.assert_array_equal(xd.cpu().numpy(), x)   # argmax leaves the logits alone


def test_sampler_ties_and_flat():
    """All-equal logits: the nucleus holds ties; ids stay in range and agree with
    the reference whenever the float64 replay is clear of boundaries."""
    ref = _ref_sampler()
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    for top_p in (0.0, 0.3, 0.9):
        for seed in (1, 2, 3):
            x = np.zeros(1000, np.float32)
            xd = torch.from_numpy(x).to(DEV)
            api.sample_dev(xd, out, 1.0, top_p, seed)
            torch.cuda.synchronize()
            got = int(out.item())
            assert 0 <= got < 1000
            xr = x.copy()
            want = ref(xr.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 1000, 1.0, top_p, seed)
            if top_p == 0.0 and _clear_of_boundaries(x, 1.0, top_p, seed):
                assert got == want, (top_p, seed, got, want)


def test_generate_sampled_matches_step_by_step(tiny_model, golden_e2e):
    """pickle_cuda_generate_sampled = forward + pickle_cuda_sample_dev with
    seed + i at each step (the chat loop's seeds); temp 0 stays greedy."""
    path, prompt = tiny_model
    m = PickleModel.from_gguf(path, max_tokens=64)
    ids0, _, _ = m.generate(prompt, 32, temp=0.0, top_p=0.9, seed=7)
    np.testing.assert_array_equal(ids0, golden_e2e["ids"][:32])
    temp, top_p, seed = 0.9, 0.95, 1234
    ids, _, pos = m.generate(prompt, 40, temp=temp, top_p=top_p, seed=seed)
    assert pos == 16 + 40
    logits, kv = m.forward(prompt, 0)
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    step = []
    for i in range(40):
        ld = torch.from_numpy(logits).to(DEV)
        api.sample_dev(ld, out, temp, top_p, seed + i)
        torch.cuda.synchronize()
        step.append(int(out.item()))
        logits, kv = m.forward([step[-1]], kv)
    m.close()
    np.testing.assert_array_equal(ids, step)
    assert len(set(step)) > 5       # sampling, not a repeated argmax
