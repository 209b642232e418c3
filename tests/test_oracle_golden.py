"""The CPU oracle against the reference's own outputs (no GPU).

Pins oracle/ref_attn_cpu.c: bit-identical to the reference's attention
block (lee-muriithi-kingori/lestramanika src/pickle_fast.c:1910-2094) on
the committed known-answer cases, and bit-identical end to end when it
serves the hook-patched pickle_fast_forward on the tiny model.
"""
import os

import numpy as np
import pytest

import oracle
from kat_cases import CASES, history, kept_steps, step_inputs


def _run_case(blk, name):
    L, H, HK, D, S, theta, seed, steps = CASES[name]
    hist = history(name)
    if hist is not None:
        kc, vc = blk.cache(0)
        kc[:len(hist[0])] = hist[0]
        vc[:len(hist[1])] = hist[1]
    keep = set(kept_steps(len(steps)))
    outs = []
    for i, (layer, pos) in enumerate(steps):
        q, k, v = step_inputs(name, i)
        ao = blk.decode(layer, pos, q, k, v)
        if i in keep:
            outs.append(ao)
    return np.stack(outs)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_kats(name, golden_kats):
    L, H, HK, D, S, theta, seed, steps = CASES[name]
    o = oracle.OracleAttn(L, H, HK, D, S, theta)
    got = _run_case(o, name)
    o.close()
    assert np.array_equal(golden_kats[name + "__steps"], np.array(kept_steps(len(steps))))
    np.testing.assert_array_equal(got, golden_kats[name])


@pytest.mark.skipif(not oracle.RefBlock.available(), reason="reference not built here")
@pytest.mark.parametrize("name", ["tiny_mha_d48", "gqa4_d128"])
def test_reference_block_reproduces_fixture(name, golden_kats):
    L, H, HK, D, S, theta, seed, steps = CASES[name]
    blk = oracle.RefBlock(L, H, HK, D, S, theta)
    got = _run_case(blk, name)
    blk.close()
    np.testing.assert_array_equal(got, golden_kats[name])


def test_rope_tables_match_reference_formula():
    # inv_freq[i] = 1/powf(theta, 2i/D) in float32 (src/pickle_fast.c:1638-1640)
    inv, s, c = oracle.rope_tables(500000.0, 128, 8)
    i = np.arange(64, dtype=np.float32)
    ref = (np.float32(1.0) / np.power(np.float32(500000.0), (2 * i).astype(np.float32) / np.float32(128))).astype(np.float32)
    np.testing.assert_allclose(inv, ref, rtol=2e-7)
    ang = inv[None, :] * np.arange(8, dtype=np.float32)[:, None]
    np.testing.assert_allclose(s, np.sin(ang.astype(np.float64)), atol=1e-7)
    np.testing.assert_allclose(c, np.cos(ang.astype(np.float64)), atol=1e-7)
    assert oracle.half_of(48) == 24 and oracle.half_of(256) == 64


def test_oracle_edge_cases():
    o = oracle.OracleAttn(1, 4, 2, 64, 4)
    q = np.ones(4 * 64, np.float32)
    kv = np.ones(2 * 64, np.float32)
    ao = o.decode(0, 0, q, kv, kv * 3)
    np.testing.assert_array_equal(ao, np.full(4 * 64, 3.0, np.float32))   # softmax over one row
    with pytest.raises(ValueError):
        o.decode(0, 4, q, kv, kv)                                            # pos >= max_seq
    with pytest.raises(ValueError):
        o.decode(1, 0, q, kv, kv)                                            # bad layer
    o.close()


@pytest.mark.skipif(not os.path.exists(oracle.e2e_binary("ref")), reason="reference not built here")
def test_reference_e2e_reproduces_fixture(tiny_model, golden_e2e, tmp_path):
    model, prompt = tiny_model
    assert list(golden_e2e["prompt"]) == list(prompt)
    r = oracle.e2e_run("ref", model, str(tmp_path / "ref.bin"), 240, prompt)
    np.testing.assert_array_equal(r["ids"], golden_e2e["ids"])
    np.testing.assert_array_equal(r["logits"], golden_e2e["logits"])


@pytest.mark.skipif(not os.path.exists(oracle.e2e_binary("oracle")), reason="oracle harness not built")
def test_oracle_serves_forward_pass_bit_exact(tiny_model, golden_e2e, tmp_path):
    """The hook-patched forward pass with the oracle as its attention block
    reproduces the unmodified reference's 240 greedy ids and final logits."""
    model, prompt = tiny_model
    r = oracle.e2e_run("oracle", model, str(tmp_path / "ora.bin"), 240, prompt,
                       dump_path=str(tmp_path / "dump.bin"))
    assert r["n_prompt"] == 16 and len(r["ids"]) == 240
    np.testing.assert_array_equal(r["ids"], golden_e2e["ids"])
    np.testing.assert_array_equal(r["margins"], golden_e2e["margins"])
    np.testing.assert_array_equal(r["logits"], golden_e2e["logits"])
    layer, pos, q, k, v, ao = oracle.read_dump(str(tmp_path / "dump.bin"), 6, 6, 48)
    assert len(layer) == 256 * 6 and pos.max() == 255
