"""End to end on the tiny model: pickle's own forward pass (hook-patched
src/pickle_fast.c) with its attention block served by the B200 shim.

North_star bar: greedy-decoded token ids identical to the unmodified
reference, per-layer attention outputs within 1e-4 relative.
"""
import os

import numpy as np
import pytest

import oracle
from gpu_util import assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda_run(tiny_model, tmp_path_factory):
    exe = oracle.e2e_binary("cuda")
    if not os.path.exists(exe):
        pytest.fail(f"{exe} is not built (python -m lestramanika_b200.build --all)")
    model, prompt = tiny_model
    d = tmp_path_factory.mktemp("e2e")
    r = oracle.e2e_run("cuda", model, str(d / "cuda.bin"), 240, prompt, dump_path=str(d / "dump.bin"))
    return r, str(d / "dump.bin")


def test_greedy_ids_identical(cuda_run, golden_e2e):
    r, _ = cuda_run
    assert r["n_prompt"] == 16
    np.testing.assert_array_equal(r["ids"], golden_e2e["ids"])


def test_final_logits_close(cuda_run, golden_e2e):
    r, _ = cuda_run
    assert_rel(r["logits"], golden_e2e["logits"], what="final logits")


def test_per_layer_attention_outputs(cuda_run):
    """Replay every (token, layer) call's inputs through the oracle and compare
    the shim's output for that call."""
    _, dump = cuda_run
    layer, pos, q, k, v, ao = oracle.read_dump(dump, 6, 6, 48)
    assert len(layer) == 256 * 6
    o = oracle.OracleAttn(6, 6, 6, 48, 256, 10000.0)
    worst = 0.0
    for i in range(len(layer)):
        ref = o.decode(int(layer[i]), int(pos[i]), q[i], k[i], v[i])
        assert_rel(ao[i], ref, what=f"call {i} layer {layer[i]} pos {pos[i]}")
    o.close()
