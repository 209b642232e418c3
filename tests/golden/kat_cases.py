"""Known-answer cases for pickle's attention block.

Each case is a model shape and a sequence of decode steps (layer, pos);
the inputs of every step (q [H*D], k [HK*D], v [HK*D], N(0, 1)) are drawn
from numpy's Philox generator keyed by (case seed, step index), so the
fixture stores only the outputs. make_golden.py produced the outputs with
the reference's own attention block (lee-muriithi-kingori/lestramanika
src/pickle_fast.c:1910-2094, compiled from its sources into oracle/_ref).
"""
import numpy as np

CASES = {
    # name: (n_layers, H, HK, D, max_seq, theta, seed, steps [(layer, pos)], kept step indices)
    "tiny_mha_d48": (2, 6, 6, 48, 40, 10000.0, 11,
                     [(0, p) for p in range(40)] + [(1, p) for p in range(3)]),
    "gqa4_d128": (1, 8, 2, 128, 48, 500000.0, 12, [(0, p) for p in range(48)]),
    "gqa8_d128": (1, 16, 2, 128, 40, 500000.0, 13, [(0, p) for p in range(40)]),
    "mha_d64": (1, 4, 4, 64, 36, 10000.0, 14, [(0, p) for p in range(36)]),
    "gqa2_d96": (1, 4, 2, 96, 36, 10000.0, 15, [(0, p) for p in range(36)]),
    # RoPE at large absolute positions; rows [0, 131032) are seeded history
    # written straight into the cache (see history()).
    "long_pos_d128": (1, 4, 1, 128, 131073, 500000.0, 16, [(0, p) for p in range(131032, 131073)]),
}

# Cache rows filled before the first step (pos-major [rows][HK][D] K and V).
HISTORY_ROWS = {"long_pos_d128": 131032}


def kept_steps(n):
    """Steps whose outputs the fixture stores: edges of the 32-row tiles and a spread."""
    keep = {0, 1, 2, n - 1, n - 2}
    for p in (15, 16, 31, 32, 33, 35, 39, 40, 47):
        if p < n:
            keep.add(p)
    keep.update(range(0, n, 7))
    return sorted(keep)


def history(case):
    """(k, v) history rows [n][HK][D] for the case, or None."""
    n = HISTORY_ROWS.get(case, 0)
    if not n:
        return None
    n_layers, H, HK, D, max_seq, theta, seed, steps = CASES[case]
    rng = np.random.Generator(np.random.Philox(key=seed, counter=[1, 0, 0, 0]))
    k = rng.standard_normal((n, HK, D), dtype=np.float32)
    v = rng.standard_normal((n, HK, D), dtype=np.float32)
    return k, v


def step_inputs(case, i):
    n_layers, H, HK, D, max_seq, theta, seed, steps = CASES[case]
    rng = np.random.Generator(np.random.Philox(key=seed, counter=[0, 0, 0, i]))
    q = rng.standard_normal(H * D, dtype=np.float32)
    k = rng.standard_normal(HK * D, dtype=np.float32)
    v = rng.standard_normal(HK * D, dtype=np.float32)
    return q, k, v
