#!/usr/bin/env python3
"""Write a small Llama GGUF with quantized projections, for the device
forward pass's parity runs against the reference's own forward
(oracle/_ref/pickle_e2e_ref loads the same file).

Mixes (every projection and the output matrix in raw GGML blocks; norms F32):
  q4_k_m: q/k/o, gate, up Q4_K; v, down, output Q6_K; token_embd F16
          (the per-tensor choice of llama.cpp's Q4_K_M files)
  q8_0:   every matrix Q8_0, token_embd F32
  q4_0:   every matrix Q4_0, token_embd F16
  f16:    every matrix F16, token_embd F16
Block scales are drawn so the dequantized weights have magnitudes of a few
hundredths, like trained weights; quants are uniform random bytes.
"""
import sys

import numpy as np

from make_tiny_llama import llama_meta, write_gguf

SHAPE = dict(n_layers=3, hidden=512, ffn=1536, n_heads=8, n_kv_heads=2, head_dim=64, vocab=4096, ctx=160)
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
BLOCK = {Q4_0: (18, 32), Q8_0: (34, 32), Q4_K: (144, 256), Q6_K: (210, 256)}
MIXES = {
    "q4_k_m": dict(q=Q4_K, k=Q4_K, v=Q6_K, o=Q4_K, gate=Q4_K, up=Q4_K, down=Q6_K, output=Q6_K, embd=F16),
    "q8_0": dict(q=Q8_0, k=Q8_0, v=Q8_0, o=Q8_0, gate=Q8_0, up=Q8_0, down=Q8_0, output=Q8_0, embd=F32),
    "q4_0": dict(q=Q4_0, k=Q4_0, v=Q4_0, o=Q4_0, gate=Q4_0, up=Q4_0, down=Q4_0, output=Q4_0, embd=F16),
    "f16": dict(q=F16, k=F16, v=F16, o=F16, gate=F16, up=F16, down=F16, output=F16, embd=F16),
}


def weight_bytes(t, out_n, in_n, rng):
    if t == F32:
        return (rng.standard_normal((out_n, in_n), dtype=np.float32) * np.float32(0.02)).tobytes()
    if t == F16:
        return (rng.standard_normal((out_n, in_n)) * 0.02).astype(np.float16).tobytes()
    bb, qk = BLOCK[t]
    nb = out_n * in_n // qk
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)

    def put_f16(off, lo, hi):
        b[:, off:off + 2] = rng.uniform(lo, hi, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if t == Q4_0:
        put_f16(0, 2e-3, 6e-3)
    elif t == Q8_0:
        put_f16(0, 1e-4, 3e-4)
    elif t == Q4_K:
        put_f16(0, 1e-4, 3e-4)
        put_f16(2, 1e-4, 3e-4)
    elif t == Q6_K:
        put_f16(208, 1e-5, 3e-5)
    return b.tobytes()


def write_model(path, mix="q4_k_m", seed=0, shape=None, tied=False, output_norm=True, embd=None):
    """tied: no output.weight (the lm_head is token_embd, which the reference
    then reads as F32); output_norm=False: no output_norm.weight; embd: the
    GGML type of token_embd instead of the mix's."""
    s = dict(SHAPE, **(shape or {}))
    m = dict(MIXES[mix])
    if embd is not None:
        m["embd"] = embd
    rng = np.random.Generator(np.random.Philox(1000 + seed))
    H, HK, D, HD, ID, VS = s["n_heads"], s["n_kv_heads"], s["head_dim"], s["hidden"], s["ffn"], s["vocab"]
    norm = lambda: (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32).tobytes()  # noqa: E731
    t = [("token_embd.weight", (VS, HD), m["embd"], weight_bytes(m["embd"], VS, HD, rng))]
    for L in range(s["n_layers"]):
        p = f"blk.{L}."
        t += [
            (p + "attn_norm.weight", (HD,), F32, norm()),
            (p + "attn_q.weight", (H * D, HD), m["q"], weight_bytes(m["q"], H * D, HD, rng)),
            (p + "attn_k.weight", (HK * D, HD), m["k"], weight_bytes(m["k"], HK * D, HD, rng)),
            (p + "attn_v.weight", (HK * D, HD), m["v"], weight_bytes(m["v"], HK * D, HD, rng)),
            (p + "attn_output.weight", (HD, H * D), m["o"], weight_bytes(m["o"], HD, H * D, rng)),
            (p + "ffn_norm.weight", (HD,), F32, norm()),
            (p + "ffn_gate.weight", (ID, HD), m["gate"], weight_bytes(m["gate"], ID, HD, rng)),
            (p + "ffn_up.weight", (ID, HD), m["up"], weight_bytes(m["up"], ID, HD, rng)),
            (p + "ffn_down.weight", (HD, ID), m["down"], weight_bytes(m["down"], HD, ID, rng)),
        ]
    if output_norm:
        t.append(("output_norm.weight", (HD,), F32, norm()))
    if not tied:
        t.append(("output.weight", (VS, HD), m["output"], weight_bytes(m["output"], VS, HD, rng)))
    meta = llama_meta(s["n_layers"], HD, ID, H, HK, D, VS, s["ctx"], theta=500000.0, name="pickle-b200-" + mix)
    write_gguf(path, meta, t)
    prng = np.random.Generator(np.random.Philox(2000 + seed))
    return [int(x) for x in prng.integers(3, VS, size=24)]


if __name__ == "__main__":
    print(write_model(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "q4_k_m"))
