#!/usr/bin/env python3
"""Write the tiny Llama GGUF v3 model used for the end-to-end parity check.

Shape (the reference's CPU-runnable configuration): dim 288, 6 layers,
6 query heads, 6 KV heads, head_dim 48, FFN hidden 768, vocab 32000,
max seq 256, RoPE theta 10000, RMSNorm eps 1e-5. Every weight is F32 drawn
N(0, 0.02) from numpy's Philox generator with the given seed.

The file layout follows the GGUF v3 writer in lee-muriithi-kingori/
lestramanika tools/make_tiny_gguf.py:56-165 (header, metadata KVs, tensor
infos, 32-byte aligned data), with two deliberate differences:
  * dims are written in GGUF order (ne[0] = the contiguous input dim), and
  * llama.vocab_size is written explicitly, because pickle_arch_detect
    otherwise falls back to the last dim of token_embd
    (src/pickle.c:1010-1021).
The data of a [out][in] weight is row-major with `in` contiguous, which is
how pickle_fast_matmul_f32 reads it.

Also returns the 16-token prompt (ids uniform in [3, 32000) from the seed).

With vocab=True the file also carries a tokenizer.ggml.* vocabulary of
32000 pieces, so the reference's own CLI (`pickle infer`, which tokenises
its prompt with pickle_tok_init / pickle_tok_encode,
src/pickle_tokenizer.c:162-470) can run the model: <unk>, <s>, </s>
(control), the 256 byte-fallback pieces <0x00>..<0xFF>, then distinct
word pieces. The weights, and so every logit, are the same either way.
"""
import struct
import sys

import numpy as np

HIDDEN, N_LAYERS, N_HEADS, N_KV_HEADS, HEAD_DIM = 288, 6, 6, 6, 48
FFN, VOCAB, CTX, THETA, EPS = 768, 32000, 256, 10000.0, 1e-5
ALIGN = 32
GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, GGUF_STR, GGUF_ARR = 4, 5, 6, 7, 8, 9


def _tensors():
    t = [("token_embd.weight", (VOCAB, HIDDEN))]
    for L in range(N_LAYERS):
        p = f"blk.{L}."
        t += [
            (p + "attn_norm.weight", (HIDDEN,)),
            (p + "attn_q.weight", (N_HEADS * HEAD_DIM, HIDDEN)),
            (p + "attn_k.weight", (N_KV_HEADS * HEAD_DIM, HIDDEN)),
            (p + "attn_v.weight", (N_KV_HEADS * HEAD_DIM, HIDDEN)),
            (p + "attn_output.weight", (HIDDEN, N_HEADS * HEAD_DIM)),
            (p + "ffn_norm.weight", (HIDDEN,)),
            (p + "ffn_gate.weight", (FFN, HIDDEN)),
            (p + "ffn_up.weight", (FFN, HIDDEN)),
            (p + "ffn_down.weight", (HIDDEN, FFN)),
        ]
    t += [("output_norm.weight", (HIDDEN,)), ("output.weight", (VOCAB, HIDDEN))]
    return t


def _s(b):
    b = b.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, meta, tensors):
    """meta: [(key, GGUF value type, value)]; tensors: [(name, shape, ggml_type,
    raw bytes)] with shape in [out][in] order (written reversed, GGUF order)."""
    head = bytearray()
    head += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    for key, typ, val in meta:
        head += _s(key) + struct.pack("<I", typ)
        if typ == GGUF_STR:
            head += _s(val)
        elif typ == GGUF_ARR:
            etyp, items = val
            head += struct.pack("<IQ", etyp, len(items))
            if etyp == GGUF_STR:
                head += b"".join(_s(x) for x in items)
            elif etyp == GGUF_F32:
                head += struct.pack(f"<{len(items)}f", *items)
            else:
                head += struct.pack(f"<{len(items)}i", *items)
        elif typ == GGUF_U32:
            head += struct.pack("<I", val)
        elif typ == GGUF_F32:
            head += struct.pack("<f", val)
        else:
            head += struct.pack("<B", 1 if val else 0)
    off = 0
    offsets = []
    for _, _, _, raw in tensors:
        offsets.append(off)
        off += len(raw)
        off += (-off) % ALIGN
    for (name, shape, gtype, _), o in zip(tensors, offsets):
        dims = tuple(reversed(shape))          # GGUF: ne[0] is the contiguous dim
        head += _s(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", gtype, o)
    head += b"\0" * ((-len(head)) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for _, _, _, raw in tensors:
            f.write(raw)
            f.write(b"\0" * ((-len(raw)) % ALIGN))


def llama_meta(n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim, vocab, ctx, theta=THETA, eps=EPS,
               name="pickle-b200-tiny"):
    return [
        ("general.architecture", GGUF_STR, "llama"),
        ("general.name", GGUF_STR, name),
        ("llama.block_count", GGUF_U32, n_layers),
        ("llama.embedding_length", GGUF_U32, hidden),
        ("llama.feed_forward_length", GGUF_U32, ffn),
        ("llama.attention.head_count", GGUF_U32, n_heads),
        ("llama.attention.head_count_kv", GGUF_U32, n_kv_heads),
        ("llama.context_length", GGUF_U32, ctx),
        ("llama.rope.dimension_count", GGUF_U32, head_dim),
        ("llama.vocab_size", GGUF_U32, vocab),
        ("llama.attention.layer_norm_rms_epsilon", GGUF_F32, eps),
        ("llama.rope.freq_base", GGUF_F32, theta),
        ("llama.tie_word_embeddings", GGUF_BOOL, False),
    ]


BOS_ID, EOS_ID, UNK_ID = 1, 2, 0


def vocab_meta(vocab=VOCAB):
    """tokenizer.ggml.* keys: control pieces, byte fallback, distinct word pieces."""
    pieces = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    types = [2, 3, 3] + [6] * 256
    pieces += ["\u2581w%05d" % i for i in range(len(pieces), vocab)]
    types += [1] * (vocab - len(types))
    scores = [0.0] * 3 + [0.0] * 256 + [-float(i) for i in range(259, vocab)]
    return [
        ("tokenizer.ggml.model", GGUF_STR, "llama"),
        ("tokenizer.ggml.tokens", GGUF_ARR, (GGUF_STR, pieces)),
        ("tokenizer.ggml.scores", GGUF_ARR, (GGUF_F32, scores)),
        ("tokenizer.ggml.token_type", GGUF_ARR, (GGUF_I32, types)),
        ("tokenizer.ggml.bos_token_id", GGUF_U32, BOS_ID),
        ("tokenizer.ggml.eos_token_id", GGUF_U32, EOS_ID),
        ("tokenizer.ggml.unknown_token_id", GGUF_U32, UNK_ID),
    ]


def write_model(path, seed=0, vocab=False):
    rng = np.random.Generator(np.random.Philox(seed))
    meta = llama_meta(N_LAYERS, HIDDEN, FFN, N_HEADS, N_KV_HEADS, HEAD_DIM, VOCAB, CTX)
    if vocab:
        meta += vocab_meta()
    tensors = _tensors()
    datas = [rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(0.02)
             for _, shape in tensors]
    write_gguf(path, meta, [(name, shape, 0, d.tobytes()) for (name, shape), d in zip(tensors, datas)])
    return prompt_ids(seed)


def prompt_ids(seed=0, n=16):
    rng = np.random.Generator(np.random.Philox(seed + 1))
    return [int(x) for x in rng.integers(3, VOCAB, size=n)]


if __name__ == "__main__":
    out = sys.argv[1] if len(sys.argv) > 1 else "/tmp/pickle_tiny.gguf"
    print(write_model(out, int(sys.argv[2]) if len(sys.argv) > 2 else 0))
