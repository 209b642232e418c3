"""Continuous batching on the GPU: requests with different prompt lengths
share one handle's cache slots, decode together each at its own position
(pickle_cuda_decode_ragged_dev), and a finished request's slot is reused by
a new one. Every output row matches a per-request oracle (the reference
block run token by token, src/pickle_fast.c:1881) within 1e-4."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_rel, normal
from lestramanika_b200 import PickleCuda, PickleError
from lestramanika_b200.slots import KVSlots

pytestmark = pytest.mark.gpu

H, HK, D, S, THETA = 8, 2, 128, 128, 10000.0
DEV = torch.device("cuda", 0)


def _tok(seed, i):
    return normal(seed, H * D, i, 1), normal(seed, HK * D, i, 2), normal(seed, HK * D, i, 3)


def test_continuous_batching_matches_per_request_oracle():
    cu = PickleCuda(1, H, HK, D, S, rope_theta=THETA, n_seqs=3)
    slots = KVSlots(cu)
    orc, n_tok = {}, {}

    def admit(req, T, seed):
        slots.admit(req)
        orc[req] = oracle.OracleAttn(1, H, HK, D, S, THETA)
        toks = [_tok(seed, i) for i in range(T)]
        q = torch.from_numpy(np.stack([t[0] for t in toks]).reshape(T, H, D)).to(DEV)
        k = torch.from_numpy(np.stack([t[1] for t in toks]).reshape(T, HK, D)).to(DEV)
        v = torch.from_numpy(np.stack([t[2] for t in toks]).reshape(T, HK, D)).to(DEV)
        ao = torch.empty((T, H, D), device=DEV)
        slots.prefill(req, 0, q, k, v, ao)
        cu.sync()
        ref = np.stack([orc[req].decode(0, i, *toks[i]) for i in range(T)])
        assert_rel(ao.cpu().numpy().reshape(T, -1), ref, what=f"prefill {req}")
        slots.advance(req, T)
        n_tok[req] = T

    def step(reqs, seed):
        toks = [_tok(seed, n_tok[r]) for r in reqs]
        q = torch.from_numpy(np.stack([t[0] for t in toks]).reshape(len(reqs), H, D)).to(DEV)
        k = torch.from_numpy(np.stack([t[1] for t in toks]).reshape(len(reqs), HK, D)).to(DEV)
        v = torch.from_numpy(np.stack([t[2] for t in toks]).reshape(len(reqs), HK, D)).to(DEV)
        ao = torch.empty((len(reqs), H, D), device=DEV)
        slots.decode(0, reqs, q, k, v, ao)
        cu.sync()
        got = ao.cpu().numpy()
        for i, r in enumerate(reqs):
            ref = orc[r].decode(0, slots.position(r), *toks[i])
            assert_rel(got[i].reshape(-1), ref, what=f"decode {r} at {slots.position(r)}")
        slots.advance(list(reqs))
        for r in reqs:
            n_tok[r] += 1

    admit("a", 20, 1)
    admit("b", 7, 2)
    admit("c", 33, 3)
    for s in range(3):
        step(["a", "b", "c"], 10 + s)
    slots.release("b")
    orc.pop("b").close()
    admit("d", 5, 4)                        # takes b's slot; b's old rows are beyond d's positions
    for s in range(3):
        step(["c", "a", "d"], 20 + s)
    for o in orc.values():
        o.close()
    cu.close()


def test_ragged_decode_at_equal_positions_equals_batch_decode():
    B, ctx = 3, 300
    cu = PickleCuda(1, H, HK, D, ctx + 1, rope_theta=THETA, n_seqs=B)
    kt, vt = cu.kv_tensors(0)
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    kt.normal_(generator=g)
    vt.normal_(generator=g)
    q = torch.randn((B, H, D), generator=g, device=DEV)
    k = torch.randn((B, HK, D), generator=g, device=DEV)
    v = torch.randn((B, HK, D), generator=g, device=DEV)
    ao1 = torch.empty((B, H, D), device=DEV)
    ao2 = torch.empty((B, H, D), device=DEV)
    cu.decode_batch_dev(0, B, ctx, q, k, v, ao1)
    pos = torch.full((B,), ctx, dtype=torch.int32, device=DEV)
    cu.decode_ragged_dev(0, pos, q, k, v, ao2)
    cu.sync()
    assert torch.equal(ao1, ao2)
    cu.close()


def test_ragged_decode_rejects_bad_positions_and_slots():
    cu = PickleCuda(1, H, HK, D, 64, rope_theta=THETA, n_seqs=2)
    q = torch.zeros((2, H, D), device=DEV)
    k = torch.zeros((2, HK, D), device=DEV)
    ao = torch.empty((2, H, D), device=DEV)
    with pytest.raises(PickleError) as e:                      # max_pos beyond the cache
        cu.decode_ragged_dev(0, torch.tensor([1, 2], dtype=torch.int32, device=DEV), q, k, k, ao, max_pos=64)
    assert e.value.code == -7
    # a position above the declared bound is skipped on the device and reported
    cu.decode_ragged_dev(0, torch.tensor([1, 9], dtype=torch.int32, device=DEV), q, k, k, ao, max_pos=5)
    with pytest.raises(PickleError) as e:
        cu.sync()
    assert e.value.code == -9
    # so is a slot outside the handle
    cu.decode_ragged_dev(0, torch.tensor([1, 2], dtype=torch.int32, device=DEV), q, k, k, ao,
                         slots=torch.tensor([0, 5], dtype=torch.int32, device=DEV), max_pos=2)
    with pytest.raises(PickleError) as e:
        cu.sync()
    assert e.value.code == -9
    # and the handle keeps working afterwards
    cu.decode_ragged_dev(0, torch.tensor([1, 2], dtype=torch.int32, device=DEV), q, k, k, ao, max_pos=2)
    cu.sync()
    cu.close()
