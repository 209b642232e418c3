"""pickle_cuda_decode_noalloc: the decode entry point for callers that cannot
let a library allocate device memory (their HBM is handed out by their own
arena, e.g. an engine that reserves it all for its KV cache, or a pickle build
that routes every allocation through pickle_alloc_t).

It must give the same outputs as the allocating entry point
pickle_cuda_decode_batch_dev (within the FP32 tolerance of the other tests,
1e-4 relative) on two calls in a row, and the CPU oracle's on the first,
through the C ABI, with the KV cache, RoPE tables, inputs and outputs all
owned by the caller and its split-KV scratch taken from the library's fixed
device array.

This file is collected last so that a stop-at-first-failure run has run every
other test before it.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_rel
from lestramanika_b200 import PickleCuda, api

pytestmark = pytest.mark.gpu


def _inputs(seed, B, H, HK, D):
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    dev = torch.device("cuda", 0)
    return (torch.randn((B, H, D), generator=g, device=dev), torch.randn((B, HK, D), generator=g, device=dev),
            torch.randn((B, HK, D), generator=g, device=dev))


@pytest.mark.parametrize("B,H,HK,D,ctx", [(2, 32, 8, 128, 3000), (1, 64, 8, 128, 5000), (3, 6, 6, 48, 200)])
def test_noalloc_matches_allocating_entry_point(B, H, HK, D, ctx):
    theta = 500000.0
    max_seq = ctx + 2
    dev = torch.device("cuda", 0)
    # Allocating path: the library's handle owns cache and tables.
    cu = PickleCuda(1, H, HK, D, max_seq, rope_theta=theta, n_seqs=B)
    kt, vt = cu.kv_tensors(0)
    g = torch.Generator(device="cuda:0")
    g.manual_seed(ctx)
    kt[:, :, :ctx].normal_(generator=g)
    vt[:, :, :ctx].normal_(generator=g)
    # No-allocation path: the caller's own copies of the cache and tables.
    k_cache = kt.clone()
    v_cache = vt.clone()
    half = min(D // 2, 64)
    _, s, c = oracle.rope_tables(theta, D, max_seq)
    rope_sin = torch.from_numpy(np.ascontiguousarray(s)).to(dev)
    rope_cos = torch.from_numpy(np.ascontiguousarray(c)).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    splits = cu.decode_plan(B, ctx)[0]
    kc0 = kt.permute(0, 2, 1, 3)[:, :ctx + 1].cpu().numpy().copy()     # pos-major copies for the oracle
    vc0 = vt.permute(0, 2, 1, 3)[:, :ctx + 1].cpu().numpy().copy()
    for step, pos in enumerate((ctx, ctx + 1)):                # two calls in a row
        q, k, v = _inputs(100 + step, B, H, HK, D)
        ao_ref = torch.empty((B, H, D), device=dev)
        ao = torch.full((B, H, D), float("nan"), device=dev)
        cu.decode_batch_dev(0, B, pos, q, k, v, ao_ref)
        api.decode_noalloc(B, H, HK, D, half, max_seq, pos, rope_sin, rope_cos, q, k, v, k_cache, v_cache, ao,
                           err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert_rel(ao.cpu().numpy(), ao_ref.cpu().numpy(), what=f"call {step} pos {pos} (splits {splits})")
        if step == 0:       # and the reference's own arithmetic (src/pickle_fast.c:1910-2094)
            ref = oracle.decode_batch(H, HK, D, pos, s[pos], c[pos], kc0, vc0, q.cpu().numpy(), k.cpu().numpy(),
                                      v.cpu().numpy())
            assert_rel(ao.cpu().numpy(), ref, what=f"call {step} vs oracle")
        np.testing.assert_array_equal(k_cache[:, :, pos].cpu().numpy(), kt[:, :, pos].cpu().numpy())
        np.testing.assert_array_equal(v_cache[:, :, pos].cpu().numpy(), vt[:, :, pos].cpu().numpy())
    cu.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    dev = torch.device("cuda", 0)
    t = torch.zeros(16, device=dev)
    with pytest.raises(api.PickleError) as e:              # 1025 * 4 > 4096 sequence/KV-head slots
        api.decode_noalloc(1025, 32, 4, 128, 64, 8, 0, t, t, t, t, t, t, t, t)
    assert e.value.code == -7
    with pytest.raises(api.PickleError) as e:              # pos >= max_seq
        api.decode_noalloc(1, 8, 8, 128, 64, 8, 8, t, t, t, t, t, t, t, t)
    assert e.value.code == -7
