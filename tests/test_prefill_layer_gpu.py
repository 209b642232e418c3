"""The attention half of a layer for a whole prompt on the device
(LayerPrefill: q/k/v GEMMs over raw GGML weights -> RoPE, cache append and
causal attention -> output-projection GEMM) against the reference's way of
doing it, one token at a time: per token, the restated matvec
(oracle/matvec.py) for q, k and v, the oracle attention block for that
position (oracle.OracleAttn, pinned to the reference's), and the matvec of
the output projection. A second prompt chunk continues from the cache the
first one filled. Bars: the F32 bar of this library (1e-4 relative to the
largest output) for F32 attention; 2e-2 with BF16 attention operands."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import BF16_ABS_TOL, assert_rel, normal
from oracle import matvec as mv
from lestramanika_b200 import PREFILL_BF16, PREFILL_F32, PickleCuda
from lestramanika_b200.prefill_layer import LayerPrefill

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("wtype", ["Q4_K", "Q8_0", "F16", "Q6_K"])
@pytest.mark.parametrize("H,HK,D,precision", [(8, 2, 64, PREFILL_F32), (4, 2, 128, PREFILL_BF16)])
def test_layer_prefill_matches_token_by_token(wtype, H, HK, D, precision):
    hidden, theta = 2048, 10000.0
    qd, kd = H * D, HK * D
    t = mv.TYPES[wtype]
    rng = np.random.default_rng(t * 31 + D)
    W = {n: mv.random_weights(t, o, i, rng) for n, (o, i) in
         {"q": (qd, hidden), "k": (kd, hidden), "v": (kd, hidden), "o": (hidden, qd)}.items()}
    shape = {"q": (qd, hidden), "k": (kd, hidden), "v": (kd, hidden), "o": (hidden, qd)}
    chunks = [(0, 100), (100, 37)]
    S = sum(c[1] for c in chunks) + 8
    cu = PickleCuda(1, H, HK, D, S, rope_theta=theta)
    lp = LayerPrefill(cu, *[(t, _dev(W[n])) for n in "qkvo"], hidden=hidden, max_tokens=128)
    o = oracle.OracleAttn(1, H, HK, D, S, theta)
    # activations scaled so that q has unit rms (attention logits of order one)
    x0 = normal(39, (4, hidden), D)
    xs = np.float32(1.0 / np.sqrt(np.mean(mv.matvec(t, W["q"], *shape["q"], x0) ** 2)))
    for ci, (pos0, T) in enumerate(chunks):
        x = normal(40 + ci, (T, hidden), D) * xs
        out = torch.empty((T, hidden), device=DEV)
        lp.run(0, pos0, _dev(x), out, precision)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        q = mv.matvec(t, W["q"], *shape["q"], x).astype(np.float32)
        k = mv.matvec(t, W["k"], *shape["k"], x).astype(np.float32)
        v = mv.matvec(t, W["v"], *shape["v"], x).astype(np.float32)
        ao = np.stack([o.decode(0, pos0 + i, q[i], k[i], v[i]) for i in range(T)])
        ref = mv.matvec(t, W["o"], *shape["o"], ao)
        tol = 1e-4 if precision == PREFILL_F32 else BF16_ABS_TOL
        assert_rel(got, ref, tol=tol, what=f"{wtype} D={D} chunk at {pos0}")
    o.close()
    cu.close()


def test_layer_prefill_rejects_long_prompt():
    cu = PickleCuda(1, 4, 2, 64, 64)
    w = (mv.TYPES["F16"], torch.zeros(256 * 512 * 2, dtype=torch.uint8, device=DEV))
    lp = LayerPrefill(cu, w, w, w, w, hidden=512, max_tokens=16)
    with pytest.raises(ValueError):
        lp.run(0, 0, torch.zeros((17, 512), device=DEV), torch.empty((17, 512), device=DEV))
    cu.close()
