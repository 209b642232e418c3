"""Helpers for the GPU parity tests (seeded inputs, tolerance checks)."""
import numpy as np

# FP32 paths: max |gpu - oracle| <= REL_TOL * max |oracle|  (north_star: 1e-4 relative).
REL_TOL = 1e-4
# BF16 tensor-core prefill: max-abs error bound (north_star: 2e-2).
BF16_ABS_TOL = 2e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def assert_rel(got, ref, tol=REL_TOL, what=""):
    e = rel_err(got, ref)
    assert e <= tol, f"{what}: relative error {e:.3e} > {tol:.1e}"


def rng(seed, *counter):
    c = list(counter) + [0] * (4 - len(counter))
    return np.random.Generator(np.random.Philox(key=seed, counter=c[:4]))


def normal(seed, shape, *counter):
    return rng(seed, *counter).standard_normal(shape, dtype=np.float32)
