"""Host side of the device forward pass, without a GPU: the GGUF reader
against the files the test writers make, arch detection with the
reference's defaults, the ctypes mirror of pickle_cuda_model_params_t
against the C header's layout (compiled here with gcc), and the tensor
lookup's errors, which come before any device call."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

import make_quant_llama as mq
import make_tiny_llama as mt
from lestramanika_b200 import api, gguf
from lestramanika_b200.model import PickleModel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_gguf_reads_the_tiny_model(tiny_model):
    path, _ = tiny_model
    meta, t = gguf.read(path)
    a = gguf.arch_detect(meta, t)
    assert (a["n_layers"], a["hidden_dim"], a["intermediate_dim"], a["n_heads"], a["n_kv_heads"], a["head_dim"],
            a["vocab_size"], a["max_seq"]) == (mt.N_LAYERS, mt.HIDDEN, mt.FFN, mt.N_HEADS, mt.N_KV_HEADS,
                                                mt.HEAD_DIM, mt.VOCAB, mt.CTX)
    assert a["rms_eps"] == np.float32(mt.EPS) and a["rope_theta"] == mt.THETA and a["tie_word_embeddings"] == 0
    typ, dims, data = t["token_embd.weight"]
    assert typ == 0 and dims == [mt.HIDDEN, mt.VOCAB]
    rng = np.random.Generator(np.random.Philox(0))
    want = rng.standard_normal(mt.VOCAB * mt.HIDDEN, dtype=np.float32) * np.float32(0.02)
    np.testing.assert_array_equal(data.view(np.float32), want)
    assert len(t) == 2 + 1 + 9 * mt.N_LAYERS


@pytest.mark.parametrize("mix", sorted(mq.MIXES))
def test_gguf_reads_quantized_blocks(tmp_path, mix):
    path = str(tmp_path / "m.gguf")
    mq.write_model(path, mix)
    meta, t = gguf.read(path)
    s, m = mq.SHAPE, mq.MIXES[mix]
    typ, dims, data = t["blk.1.ffn_down.weight"]
    assert typ == m["down"] and dims == [s["ffn"], s["hidden"]]
    assert data.nbytes == s["hidden"] * api_row_bytes(typ, s["ffn"])
    assert gguf.arch_detect(meta, t)["rope_theta"] == 500000.0


def api_row_bytes(typ, n):
    bb, be = gguf.BLOCK[typ]
    return n // be * bb


def test_arch_detect_defaults():
    meta = {"llama.block_count": 2, "llama.embedding_length": 64, "llama.feed_forward_length": 128,
            "llama.attention.head_count": 4}
    t = {"token_embd.weight": (0, [64, 1000], None)}
    a = gguf.arch_detect(meta, t)
    # src/pickle.c:1001-1021: HK = H, ctx 2048, eps 1e-5, theta 10000, D = hidden / H, vocab from the last dim
    assert (a["n_kv_heads"], a["max_seq"], a["head_dim"], a["vocab_size"]) == (4, 2048, 16, 1000)
    assert a["rms_eps"] == 1e-5 and a["rope_theta"] == 10000.0
    with pytest.raises(gguf.GGUFError):
        gguf.arch_detect({}, t)


def test_gguf_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + bytes(16))
    with pytest.raises(gguf.GGUFError):
        gguf.read(str(p))
    p.write_bytes(b"NOPE" + bytes(20))
    with pytest.raises(gguf.GGUFError):
        gguf.read(str(p))


def test_gguf_rejects_truncated_files(tmp_path, tiny_model):
    path, _ = tiny_model
    data = open(path, "rb").read()
    for cut in (10, 200, 3000, len(data) - 100):     # in the header, the tensor infos, the data
        p = tmp_path / f"cut{cut}.gguf"
        p.write_bytes(data[:cut])
        with pytest.raises(gguf.GGUFError):
            gguf.read(str(p))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_model_params_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    fields = ["rope_inv_freq", "max_tokens", "prefill_precision", "weights_on_device", "token_embd", "output_norm",
              "output", "layers", "n_seqs"]
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include <stdint.h>\n#include \"pickle_cuda.h\"\n"
                   "int main(void){printf(\"%zu %zu %zu\", sizeof(pickle_cuda_tensor_t),"
                   " offsetof(pickle_cuda_tensor_t, nbytes), sizeof(pickle_cuda_model_params_t));"
                   + "".join(f"printf(\" %zu\", offsetof(pickle_cuda_model_params_t, {f}));" for f in fields)
                   + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), "-o", str(exe), str(src)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [ctypes.sizeof(api.Tensor), api.Tensor.nbytes.offset, ctypes.sizeof(api.ModelParams)] + \
        [getattr(api.ModelParams, f).offset for f in fields]
    assert got == want


def test_model_missing_tensor_raises_arch(tmp_path):
    path = str(tmp_path / "m.gguf")
    mq.write_model(path, "q8_0")
    meta, t = gguf.read(path)
    tensors = {n: (typ, d) for n, (typ, dims, d) in t.items() if n != "blk.2.ffn_up.weight"}
    with pytest.raises(api.PickleError) as e:
        PickleModel(tensors, gguf.arch_detect(meta, t))
    assert e.value.code == -8 and "blk.2.ffn_up.weight" in str(e.value)
