"""Decode parity on the GPU: the C ABI against the oracle / the reference's KATs.

Bar (north_star): 1e-4 relative for the FP32 decode path.
"""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_rel, normal
from kat_cases import CASES, history, kept_steps, step_inputs
from lestramanika_b200 import PickleCuda, PickleError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(CASES))
def test_decode_matches_reference_kats(name, golden_kats):
    """Host-buffer entry point (what the hooked pickle_fast_forward calls), step
    by step, against the reference block's own outputs."""
    L, H, HK, D, S, theta, seed, steps = CASES[name]
    cu = PickleCuda(L, H, HK, D, S, rope_theta=theta)
    hist = history(name)
    if hist is not None:
        cu.kv_write(0, 0, 0, hist[0], hist[1])
    keep = kept_steps(len(steps))
    got = []
    for i, (layer, pos) in enumerate(steps):
        q, k, v = step_inputs(name, i)
        ao = cu.attn_decode(layer, pos, q, k, v)
        if i in keep:
            got.append(ao)
    cu.close()
    for j, i in enumerate(keep):
        assert_rel(got[j], golden_kats[name][j], what=f"{name} step {i}")


def _cache_case(B, H, HK, D, ctx, seed, theta=500000.0):
    """Seeded N(0,1) caches (pos-major, as the reference holds them) and new q/k/v."""
    max_seq = ctx + 1
    kc = np.zeros((B, max_seq, HK, D), np.float32)
    vc = np.zeros((B, max_seq, HK, D), np.float32)
    kc[:, :ctx] = normal(seed, (B, ctx, HK, D), 1)
    vc[:, :ctx] = normal(seed, (B, ctx, HK, D), 2)
    q = normal(seed, (B, H, D), 3)
    k = normal(seed, (B, HK, D), 4)
    v = normal(seed, (B, HK, D), 5)
    return kc, vc, q, k, v


def _run_batch(B, H, HK, D, ctx, seed, theta=500000.0):
    kc, vc, q, k, v = _cache_case(B, H, HK, D, ctx, seed, theta)
    max_seq = ctx + 1
    cu = PickleCuda(1, H, HK, D, max_seq, rope_theta=theta, n_seqs=B)
    for b in range(B):
        cu.kv_write(0, b, 0, kc[b, :ctx], vc[b, :ctx])
    dev = torch.device("cuda", 0)
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    ao = torch.empty((B, H, D), dtype=torch.float32, device=dev)
    cu.decode_batch_dev(0, B, ctx, qd, kd, vd, ao)
    cu.sync()
    got = ao.cpu().numpy()
    kt, vt = cu.kv_tensors(0)
    new_k = kt[:, :, ctx, :].cpu().numpy()
    new_v = vt[:, :, ctx, :].cpu().numpy()
    splits = cu.decode_plan(B, ctx)[0]
    cu.close()
    _, s, c = oracle.rope_tables(theta, D, max_seq)
    ref = oracle.decode_batch(H, HK, D, ctx, s[ctx], c[ctx], kc, vc, q, k, v)
    return got, ref, new_k, kc[:, ctx], new_v, vc[:, ctx], splits


@pytest.mark.parametrize("B,H,HK,D,ctx", [
    (1, 32, 8, 128, 4096),    # Llama-3-8B decode, B=1 (full size)
    (8, 32, 8, 128, 4096),    # B=8 (full size)
    (3, 32, 8, 128, 777),     # ragged batch / context
    (2, 64, 8, 128, 2049),    # Llama-3-70B group size 8
    (2, 6, 6, 48, 255),       # tiny model shape
    (2, 8, 4, 64, 100),       # G=2, D=64
    (1, 16, 2, 256, 300),     # D=256
])
def test_batch_decode_matches_oracle(B, H, HK, D, ctx):
    got, ref, nk, rk, nv, rv, splits = _run_batch(B, H, HK, D, ctx, seed=B * 1000 + ctx)
    assert_rel(got, ref, what=f"B={B} H={H} HK={HK} D={D} ctx={ctx} splits={splits}")
    np.testing.assert_allclose(nk, rk, rtol=0, atol=1e-5)     # appended, rotated k
    np.testing.assert_array_equal(nv, rv)                      # appended v


def test_batch_decode_b64_full_size():
    """Llama-3-8B decode at the headline batch (B=64, ctx 4096)."""
    got, ref, nk, rk, nv, rv, splits = _run_batch(64, 32, 8, 128, 4096, seed=64)
    assert_rel(got, ref, what=f"B=64 splits={splits}")
    np.testing.assert_array_equal(nv, rv)


@pytest.mark.parametrize("ctx", [0, 1, 2, 31, 32, 33, 63, 64, 65, 95, 96, 97, 127, 128, 129, 200])
def test_decode_tile_and_split_edges(ctx):
    got, ref, *_ = _run_batch(1, 32, 8, 128, ctx, seed=7 + ctx)
    assert_rel(got, ref, what=f"ctx={ctx}")


def test_decode_long_context_full_size():
    """Long-context decode (ctx 131072, B=1, 32 heads over 8 KV heads): the
    full-size single-GPU case of the sequence-sharded configuration."""
    got, ref, nk, rk, nv, rv, splits = _run_batch(1, 32, 8, 128, 131072, seed=131072)
    assert_rel(got, ref, what=f"ctx=131072 splits={splits}")


def test_zero_history_sum_is_more_exact_than_sequential():
    """131K identical softmax terms (all-zero history): the reference's
    sequential F32 sum drifts by ~1e-3 relative; the split/tile sums here
    stay within 1e-5 of a float64 evaluation."""
    H, HK, D, ctx = 4, 1, 128, 131072
    cu = PickleCuda(1, H, HK, D, ctx + 1, rope_theta=500000.0)
    q, k, v = normal(3, H * D, 1), normal(3, HK * D, 2), normal(3, HK * D, 3)
    got = cu.attn_decode(0, ctx, q, k, v).reshape(H, D).astype(np.float64)
    cu.close()
    _, s, c = oracle.rope_tables(500000.0, D, ctx + 1)
    qr = oracle.rope_apply(q.reshape(H, D), D, s[ctx], c[ctx]).astype(np.float64)
    kr = oracle.rope_apply(k.reshape(HK, D), D, s[ctx], c[ctx]).astype(np.float64)
    sc = (qr @ kr[0]) * np.float64(np.float32(1.0) / np.sqrt(np.float32(D)))
    m = np.maximum(sc, 0.0)
    w = np.exp(sc - m)
    ref64 = (w / (ctx * np.exp(-m) + w))[:, None] * v.astype(np.float64)[None, :]
    assert float(np.max(np.abs(got - ref64)) / np.max(np.abs(ref64))) <= 1e-5


def test_decode_errors():
    cu = PickleCuda(2, 8, 2, 128, 16)
    q = np.zeros(8 * 128, np.float32)
    k = np.zeros(2 * 128, np.float32)
    with pytest.raises(PickleError) as e:
        cu.attn_decode(0, 16, q, k, k)
    assert e.value.code == -7                       # PICKLE_ERR_RANGE (src/pickle_fast.c:1885)
    with pytest.raises(PickleError) as e:
        cu.attn_decode(2, 0, q, k, k)
    assert e.value.code == -6                       # PICKLE_ERR_ARG
    cu.close()
    with pytest.raises(PickleError) as e:
        PickleCuda(1, 6, 4, 128, 16)                # H % HK != 0
    assert e.value.code == -6
    with pytest.raises(PickleError) as e:
        PickleCuda(1, 8, 8, 50, 16)                 # D not a multiple of 4
    assert e.value.code == -6


def test_sequential_steps_reuse_device_cache():
    """Many steps through the host API: the device cache built by earlier
    appends is what later steps attend over (GQA 4, two layers)."""
    H, HK, D, S = 8, 2, 128, 100
    cu = PickleCuda(2, H, HK, D, S, rope_theta=10000.0)
    o = oracle.OracleAttn(2, H, HK, D, S, 10000.0)
    for pos in range(S):
        for layer in range(2):
            q = normal(99, H * D, pos, layer, 1)
            k = normal(99, HK * D, pos, layer, 2)
            v = normal(99, HK * D, pos, layer, 3)
            assert_rel(cu.attn_decode(layer, pos, q, k, v), o.decode(layer, pos, q, k, v),
                       what=f"pos={pos} layer={layer}")
    cu.close()
    o.close()


def _rope_np(x, half, sn, cs):
    """NeoX rotation of the first 2*half elements (src/pickle_fast.c:1917-1924), float64."""
    y = x.astype(np.float64).copy()
    lo, hi = x[..., :half].astype(np.float64), x[..., half:2 * half].astype(np.float64)
    y[..., :half] = cs * lo - sn * hi
    y[..., half:2 * half] = sn * lo + cs * hi
    return y


def test_partial_rotary_half_not_multiple_of_four():
    """An explicit rotary width of 30 pairs (not a multiple of four) takes the
    element-wise RoPE loads; checked against a float64 restatement."""
    B, H, HK, D, ctx, half, theta = 2, 8, 2, 64, 300, 30, 10000.0
    dev = torch.device("cuda", 0)
    cu = PickleCuda(1, H, HK, D, ctx + 1, half=half, rope_theta=theta, n_seqs=B)
    kc = normal(5, (B, HK, ctx, D), 1)
    vc = normal(5, (B, HK, ctx, D), 2)
    kt, vt = cu.kv_tensors(0)
    kt[:, :, :ctx] = torch.from_numpy(kc).to(dev)
    vt[:, :, :ctx] = torch.from_numpy(vc).to(dev)
    q, k, v = normal(5, (B, H, D), 3), normal(5, (B, HK, D), 4), normal(5, (B, HK, D), 5)
    ao = torch.empty((B, H, D), device=dev)
    cu.decode_batch_dev(0, B, ctx, *(torch.from_numpy(x).to(dev) for x in (q, k, v)), ao)
    cu.sync()
    got = ao.cpu().numpy()
    cu.close()
    inv = (1.0 / np.power(np.float32(theta), np.arange(half, dtype=np.float32) * 2 / np.float32(D))).astype(np.float32)
    ang = (inv * np.float32(ctx)).astype(np.float64)
    sn, cs = np.sin(ang), np.cos(ang)
    qr, kr = _rope_np(q, half, sn, cs), _rope_np(k, half, sn, cs)
    G = H // HK
    ref = np.empty((B, H, D))
    for b in range(B):
        for h in range(H):
            kv = h // G
            keys = np.concatenate([kc[b, kv].astype(np.float64), kr[b, kv][None]])
            vals = np.concatenate([vc[b, kv].astype(np.float64), v[b, kv].astype(np.float64)[None]])
            sc = keys @ qr[b, h] / np.sqrt(D)
            w = np.exp(sc - sc.max())
            ref[b, h] = (w / w.sum()) @ vals
    assert_rel(got, ref, what="half=30")


def test_decode_rejects_unaligned_rows():
    """q / k / v / output rows move as 16-byte vectors: a pointer off a
    16-byte boundary is an argument error, not a device fault."""
    dev = torch.device("cuda", 0)
    B, H, HK, D = 1, 8, 2, 64
    cu = PickleCuda(1, H, HK, D, 16, n_seqs=B)
    buf = torch.zeros(B * H * D + 1, device=dev)
    q_bad = buf[1:].view(B, H, D)
    k = torch.zeros((B, HK, D), device=dev)
    ao = torch.empty((B, H, D), device=dev)
    with pytest.raises(PickleError) as e:
        cu.decode_batch_dev(0, B, 3, q_bad, k, k, ao)
    assert e.value.code == -6
    out_bad = torch.empty(B * H * D + 1, device=dev)[1:].view(B, H, D)
    with pytest.raises(PickleError) as e:
        cu.decode_batch_dev(0, B, 3, torch.zeros((B, H, D), device=dev), k, k, out_bad)
    assert e.value.code == -6
    cu.close()


def _handle_with(env, *args, **kw):
    """A handle created with the given PICKLE_CUDA_* knobs set (read at creation)."""
    import os
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        return PickleCuda(*args, **kw)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


@pytest.mark.parametrize("B,H,HK,D,ctx", [
    (1, 32, 8, 128, 4096),    # 37 splits
    (2, 64, 8, 128, 2049),    # G=8
    (8, 32, 8, 128, 4096),    # two waves
    (2, 6, 6, 48, 255),       # D=48, G=1
    (1, 16, 2, 256, 300),     # D=256
])
def test_dependent_launch_agrees_bit_for_bit(B, H, HK, D, ctx):
    """The split kernel is launched as a programmatic dependent of the kernel
    before it (griddepcontrol.wait before its first global access). Steps
    that chain on one another through the cache (each appends the row the
    next attends over) must give the same bits as plain launches
    (PICKLE_CUDA_PDL=0), eagerly and in graph replay."""
    dev = torch.device("cuda", 0)
    kc, vc, q, k, v = _cache_case(B, H, HK, D, ctx, seed=ctx + 17)
    handles = [_handle_with(env, 1, H, HK, D, ctx + 8, rope_theta=500000.0, n_seqs=B)
               for env in ({}, {"PICKLE_CUDA_PDL": "0"})]
    for cu in handles:
        for b in range(B):
            cu.kv_write(0, b, 0, kc[b, :ctx], vc[b, :ctx])
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    outs = [[] for _ in handles]
    # Back-to-back steps with different split counts; step j + 1 attends the
    # row step j appended.
    steps = [(B, ctx), (B, ctx + 1), (max(1, B // 2), ctx + 2), (1, 33), (B, ctx + 3)]
    for i, cu in enumerate(handles):
        for n, p in steps:
            ao = torch.empty((n, H, D), dtype=torch.float32, device=dev)
            cu.decode_batch_dev(0, n, p, qd[:n], kd[:n], vd[:n], ao)
            outs[i].append(ao)
        cu.sync()
    for j, (n, p) in enumerate(steps):
        splits = handles[0].decode_plan(n, p)[0]
        assert torch.equal(outs[0][j], outs[1][j]), f"step {j} (n={n}, pos={p}, splits={splits})"
    # The last step again (it re-appends the same row, so the cache no longer
    # changes), twice per graph, replayed.
    cu = handles[0]
    n, p = steps[-1]
    ao = torch.empty((n, H, D), dtype=torch.float32, device=dev)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        cu.decode_batch_dev(0, n, p, qd, kd, vd, ao, stream=st)
        st.synchronize()
        with torch.cuda.graph(g, stream=st):
            cu.decode_batch_dev(0, n, p, qd, kd, vd, ao, stream=st)
            cu.decode_batch_dev(0, n, p, qd, kd, vd, ao, stream=st)
    for rep in range(3):
        ao.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ao, outs[1][-1]), f"graph replay {rep}"
    del g
    for cu in handles:
        cu.close()
    ref = _run_batch(B, H, HK, D, ctx, seed=ctx + 17)[1]
    assert_rel(outs[0][0].cpu().numpy(), ref, what=f"B={B} D={D} ctx={ctx}")
