"""The whole forward pass on the device (pickle_cuda_model_*: embedding,
norms, projections, attention block, SwiGLU, lm_head, greedy argmax)
against the reference's own forward.

* The tiny F32 Llama (tests/golden/make_tiny_llama.py): the 240 greedy ids
  and final logits that the unmodified reference produced
  (tests/golden/tiny_e2e_seed0.npz), through pickle_cuda_generate, through
  step-by-step pickle_cuda_forward calls, and with the prompt split into
  chunks.
* Small Llamas with quantized projections (tests/golden/make_quant_llama.py:
  a Q4_K_M-like mix, Q8_0, Q4_0, F16; tied embeddings; no final norm;
  quantized token embeddings, tied and untied): the
  reference's own forward (oracle/_ref/pickle_e2e_ref, the unmodified
  src/pickle_fast.c) run on the same GGUF file.

* Continuous batching through the model (n_seqs cache slots,
  pickle_cuda_forward_slot / pickle_cuda_forward_batch_dev): each request's
  ids and each row's logits against the single-sequence path.

Bars: greedy ids identical; final logits within 1e-4 of the largest logit.
"""
import os

import numpy as np
import pytest
import torch

import make_quant_llama as mq
import oracle
from gpu_util import BF16_ABS_TOL, assert_rel
from lestramanika_b200 import PREFILL_BF16, PickleError, api
from lestramanika_b200.model import PickleModel

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def tiny(tiny_model):
    path, prompt = tiny_model
    m = PickleModel.from_gguf(path, max_tokens=64)
    yield m, prompt
    m.close()


def test_generate_matches_reference_ids(tiny, golden_e2e):
    m, prompt = tiny
    ids, logits, pos = m.generate(prompt, 240)
    np.testing.assert_array_equal(ids, golden_e2e["ids"])
    assert pos == 16 + 240
    assert_rel(logits, golden_e2e["logits"], what="final logits")


def test_generate_with_prompt_chunks(tiny_model, golden_e2e):
    path, prompt = tiny_model
    m = PickleModel.from_gguf(path, max_tokens=5)      # prompt runs as 5 + 5 + 5 + 1
    ids, _, pos = m.generate(prompt, 64)
    np.testing.assert_array_equal(ids, golden_e2e["ids"][:64])
    assert pos == 16 + 64
    m.close()


def test_weights_on_device_unfused(tiny_model, golden_e2e):
    """Weights given as separate device tensors (weights_on_device): no two
    are back to back, so q, k, v and gate, up run as separate projections."""
    from lestramanika_b200 import gguf
    path, prompt = tiny_model
    meta, t = gguf.read(path)
    tensors = {n: (typ, torch.from_numpy(np.array(d)).to(DEV)) for n, (typ, dims, d) in t.items()}
    m = PickleModel(tensors, gguf.arch_detect(meta, t), max_tokens=64)
    ids, logits, pos = m.generate(prompt, 48)
    m.close()
    np.testing.assert_array_equal(ids, golden_e2e["ids"][:48])
    assert pos == 16 + 48


def test_forward_step_by_step(tiny, golden_e2e):
    """pickle_fast_forward's calling convention: the prompt, then one id at a time."""
    m, prompt = tiny
    logits, pos = m.forward(prompt, 0)
    assert pos == 16
    for i in range(24):
        nxt = int(np.argmax(logits))
        assert nxt == golden_e2e["ids"][i], i
        logits, pos = m.forward([nxt], pos)
    assert pos == 16 + 24


def test_stop_at_eos(tiny, golden_e2e):
    m, prompt = tiny
    g = golden_e2e["ids"]
    k = 5                                   # first occurrence of this id
    assert g[k] not in g[:k]
    ids, logits, pos = m.generate(prompt, 240, eos_id=int(g[k]))
    np.testing.assert_array_equal(ids, g[:k + 1])
    assert pos == 16 + k                    # the eos id is not forwarded
    assert int(np.argmax(logits)) == g[k]   # the logits it was taken from


def test_generate_stops_at_full_cache(tiny, golden_e2e):
    m, prompt = tiny
    ids, _, pos = m.generate(prompt, 400)   # max_seq 256: 240 forwards fit after the prompt
    assert len(ids) == 241 and pos == 256
    np.testing.assert_array_equal(ids[:240], golden_e2e["ids"])


def test_forward_dev_and_argmax(tiny):
    m, prompt = tiny
    ref, _ = m.forward(prompt, 0)
    tok = torch.tensor(prompt, dtype=torch.int32, device=DEV)
    logits = torch.empty(m.VS, device=DEV)
    nxt = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    s = torch.cuda.Stream()
    m.forward_dev(tok, 0, logits, nxt, stream=s)
    m.sync(stream=s)
    got = logits.cpu().numpy()
    np.testing.assert_array_equal(got, ref)         # same kernels, same inputs
    assert int(nxt.item()) == int(np.argmax(ref))


def test_forward_errors(tiny):
    m, prompt = tiny
    with pytest.raises(PickleError) as e:
        m.forward([5, m.VS], 0)
    assert e.value.code == -7
    with pytest.raises(PickleError) as e:
        m.forward([1, 2, 3], 254)                   # positions 254..256, max_seq 256
    assert e.value.code == -7
    with pytest.raises(PickleError) as e:
        m.forward([-1], 0)
    assert e.value.code == -7
    # a device-side id out of range is reported by the sync, and the model stays usable
    bad = torch.tensor([m.VS + 3], dtype=torch.int32, device=DEV)
    logits = torch.empty(m.VS, device=DEV)
    m.forward_dev(bad, 0, logits)
    with pytest.raises(PickleError) as e:
        m.sync()
    assert e.value.code == -7
    _, pos = m.forward(prompt, 0)
    assert pos == 16


def _argmax_ref(x):
    # pickle_fast_argmax (src/pickle_fast.c:2186-2194)
    best, bv = 0, x[0]
    for i in range(1, len(x)):
        if x[i] > bv:
            best, bv = i, x[i]
    return best


@pytest.mark.parametrize("case", ["ties", "nan_first", "nan_inside", "all_neg_inf", "neg_zero"])
def test_argmax_edge_cases(tiny, case):
    """pickle_cuda_argmax_dev against the reference's scan (ties, NaNs, -inf, -0)."""
    m, _ = tiny
    rng = np.random.default_rng(3)
    x = rng.standard_normal(m.VS).astype(np.float32)
    if case == "ties":
        x[[100, 7000, 31999]] = 9.0
    elif case == "nan_first":
        x[0] = np.nan
    elif case == "nan_inside":
        x[[5, 500]] = np.nan
        x[20000] = 50.0
    elif case == "all_neg_inf":
        x[:] = -np.inf
    elif case == "neg_zero":
        x[:] = -1.0
        x[10], x[11] = -0.0, 0.0
    xd = torch.from_numpy(x).to(DEV)
    out = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    api.argmax_dev(xd, out)
    torch.cuda.synchronize()
    assert int(out.item()) == _argmax_ref(x), case


@pytest.fixture(scope="module")
def quant_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("quant")


@pytest.mark.parametrize("mix,opts", [("q4_k_m", {}), ("q8_0", {}), ("q4_0", {}), ("f16", {}),
                                      ("q8_0", {"tied": True}), ("q4_k_m", {"output_norm": False}),
                                      # quantized token_embd: an F32 table at load, as the reference's state init
                                      ("q4_k_m", {"embd": mq.Q6_K}), ("q4_k_m", {"embd": mq.Q4_K}),
                                      ("q8_0", {"tied": True, "embd": mq.Q8_0}),
                                      ("q4_0", {"tied": True, "embd": mq.Q4_0})])
def test_quantized_models_match_reference(quant_dir, mix, opts):
    exe = oracle.e2e_binary("ref")
    if not os.path.exists(exe):
        pytest.fail(f"{exe} is not built (python -m lestramanika_b200.build --all)")
    tag = mix + "".join(f"_{k}{v}" for k, v in opts.items())
    path = str(quant_dir / f"{tag}.gguf")
    prompt = mq.write_model(path, mix, **opts)
    ref = oracle.e2e_run("ref", path, str(quant_dir / f"{tag}.bin"), 48, prompt)
    m = PickleModel.from_gguf(path, max_tokens=32)
    ids, logits, pos = m.generate(prompt, 48)
    m.close()
    np.testing.assert_array_equal(ids, ref["ids"])
    assert pos == len(prompt) + 48
    assert_rel(logits, ref["logits"], what=f"{tag} final logits")


def test_bf16_prefill_logits(quant_dir):
    """BF16 attention operands for the prompt (PICKLE_CUDA_PREFILL_BF16, the
    tensor-core prefill, which takes head_dim 128 prompts starting at
    position 0): the prompt's logits stay within the BF16 bar (2e-2 of the
    largest) of the F32 path, which matches the reference."""
    path = str(quant_dir / "bf16.gguf")
    prompt = mq.write_model(path, "q4_k_m", seed=1, shape=dict(n_heads=4, n_kv_heads=2, head_dim=128))
    m32 = PickleModel.from_gguf(path, max_tokens=32)
    m16 = PickleModel.from_gguf(path, max_tokens=32, precision=PREFILL_BF16)
    l32, _ = m32.forward(prompt, 0)
    l16, _ = m16.forward(prompt, 0)
    m32.close()
    m16.close()
    assert_rel(l16, l32, tol=BF16_ABS_TOL, what="bf16 prompt logits")


def _prompts(n, vocab, seed=11):
    rng = np.random.default_rng(seed)
    return [[int(t) for t in rng.integers(3, vocab, size=int(rng.integers(5, 21)))] for _ in range(n)]


def test_generate_batch_matches_single(tiny, tiny_model, golden_e2e):
    """Continuous batching through the whole model: 5 requests on 3 cache
    slots (later prompts are admitted into the slots earlier ones free);
    every request gets the ids that a single-sequence generate gives, and the
    golden prompt gets the reference's."""
    single, prompt = tiny
    path, _ = tiny_model
    prompts = [prompt] + _prompts(4, single.VS)
    n_gen = [30, 30, 30, 30, 30]
    mb = PickleModel.from_gguf(path, max_tokens=64, n_seqs=3)
    got = mb.generate_batch(prompts, 30)
    np.testing.assert_array_equal(got[0], golden_e2e["ids"][:30])
    for i, p in enumerate(prompts):
        want, _, _ = single.generate(p, n_gen[i])
        np.testing.assert_array_equal(got[i], want, err_msg=f"request {i}")
    # with an eos id: each request stops after its first occurrence
    eos = int(golden_e2e["ids"][5])
    got = mb.generate_batch(prompts, 30, eos_id=eos)
    for i, p in enumerate(prompts):
        want, _, _ = single.generate(p, 30, eos_id=eos)
        np.testing.assert_array_equal(got[i], want, err_msg=f"request {i} with eos")
    mb.close()


def test_forward_batch_rows_match_single_steps(quant_dir):
    """One batched decode step of 12 sequences (more than 8 rows: the
    projections run as GEMMs) on a Q4_K_M-like model: each row's logits
    equal that sequence's own step within the library's 1e-4 bar."""
    path = str(quant_dir / "batch.gguf")
    mq.write_model(path, "q4_k_m", seed=2)
    n = 12
    mb = PickleModel.from_gguf(path, max_tokens=32, n_seqs=n)
    ms = PickleModel.from_gguf(path, max_tokens=32)
    prompts = _prompts(n, mb.VS, seed=5)
    toks = [int(t) for t in np.random.default_rng(6).integers(3, mb.VS, size=n)]
    slots = list(range(n))[::-1]                       # slots in another order than the rows
    for p, s in zip(prompts, slots):
        mb.forward_slot(s, p, 0)
    host = np.array([toks, [len(p) for p in prompts], slots], np.int32)
    d = torch.from_numpy(host).to(DEV)
    logits = torch.empty((n, mb.VS), device=DEV)
    nxt = torch.empty(n, dtype=torch.int32, device=DEV)
    mb.forward_batch_dev(d[0], d[1], d[2], int(host[1].max()), logits, nxt)
    mb.sync()
    got = logits.cpu().numpy()
    for i, p in enumerate(prompts):
        ms.forward(p, 0)
        want, _ = ms.forward([toks[i]], len(p))
        assert_rel(got[i], want, what=f"row {i}")
        assert int(nxt[i].item()) == int(np.argmax(got[i]))
    with pytest.raises(PickleError) as e:
        mb.forward_slot(n, prompts[0], 0)
    assert e.value.code == -7
    with pytest.raises(PickleError) as e:
        ms.forward_batch_dev(d[0], d[1], d[2], int(host[1].max()), logits, nxt)   # 12 rows, 1 slot
    assert e.value.code == -7
    mb.close()
    ms.close()
