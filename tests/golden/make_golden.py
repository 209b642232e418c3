#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from the reference itself.

Needs oracle/_ref built from the reference sources (`make -C oracle ref`),
i.e. it runs where the reference tree is mounted. Writes:
  attn_block_kats.npz  - outputs of the reference's own attention block
                         (oracle/_ref/libref_attn_block.so) on the
                         kat_cases.py inputs, at the kept steps;
  tiny_e2e_seed0.npz   - prompt, greedy ids (240), per-step top-2 margins
                         and final logits of the unmodified reference
                         forward pass (oracle/_ref/pickle_e2e_ref) on the
                         make_tiny_llama.py model, seed 0.
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import oracle  # noqa: E402
from kat_cases import CASES, history, kept_steps, step_inputs  # noqa: E402
import make_tiny_llama  # noqa: E402


def make_kats():
    out = {}
    for name, (L, H, HK, D, S, theta, seed, steps) in CASES.items():
        blk = oracle.RefBlock(L, H, HK, D, S, theta)
        hist = history(name)
        if hist is not None:
            kc, vc = blk.cache(0)
            kc[:len(hist[0])] = hist[0]
            vc[:len(hist[1])] = hist[1]
        keep = set(kept_steps(len(steps)))
        aos = []
        for i, (layer, pos) in enumerate(steps):
            q, k, v = step_inputs(name, i)
            ao = blk.decode(layer, pos, q, k, v)
            if i in keep:
                aos.append(ao)
        blk.close()
        out[name] = np.stack(aos)
        out[name + "__steps"] = np.array(sorted(keep), np.int32)
    np.savez_compressed(os.path.join(HERE, "attn_block_kats.npz"), **out)


def make_e2e():
    with tempfile.TemporaryDirectory() as td:
        model = os.path.join(td, "tiny.gguf")
        prompt = make_tiny_llama.write_model(model, 0)
        r = oracle.e2e_run("ref", model, os.path.join(td, "out.bin"), 240, prompt)
    np.savez_compressed(os.path.join(HERE, "tiny_e2e_seed0.npz"), prompt=np.array(prompt, np.int32),
                        ids=r["ids"], margins=r["margins"], logits=r["logits"])


if __name__ == "__main__":
    make_kats()
    make_e2e()
    print("golden fixtures written to", HERE)
