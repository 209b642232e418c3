"""The sharded decodes with the exchange fused into the merge launch
(pickle_cuda_decode_gather_dev, pickle_cuda_decode_seqshard_dev), on one GPU:

* with one rank, the data path - split partials, the fused merge, the
  epoch-tagged stores into the exchange buffer and the assembly of the
  output from it - must reproduce the
  unsharded decode and the oracle (src/pickle_fast.c:1910-2094), on calls in
  a row and from a replayed CUDA graph;
* failure detection: a rank whose peer never arrives gives up after the
  exchange's bounded wait, reports PICKLE_ERR_DEVICE, marks the exchange
  broken, and the GPU still runs a correct decode afterwards. The peer is a
  second exchange object that never launches anything (a flag nothing sets:
  no fault, no hang).
The two-process form on two GPUs is in tests/mp_xchg_worker.py."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_rel, normal
from lestramanika_b200 import PickleCuda
from lestramanika_b200.api import SHARD_HEADS, SHARD_SEQ, PeerExchange, PickleError, decode_xchg_bytes

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _handle_with_cache(B, H, HK, D, ctx, seed, theta=500000.0):
    kc = np.zeros((B, ctx + 1, HK, D), np.float32)
    vc = np.zeros((B, ctx + 1, HK, D), np.float32)
    kc[:, :ctx] = normal(seed, (B, ctx, HK, D), 1)
    vc[:, :ctx] = normal(seed, (B, ctx, HK, D), 2)
    cu = PickleCuda(1, H, HK, D, ctx + 2, rope_theta=theta, n_seqs=B)
    for b in range(B):
        cu.kv_write(0, b, 0, kc[b, :ctx], vc[b, :ctx])
    return cu, kc, vc


def _oracle(H, HK, D, pos, kc, vc, q, k, v, theta=500000.0):
    _, s, c = oracle.rope_tables(theta, D, pos + 1)
    return oracle.decode_batch(H, HK, D, pos, s[pos], c[pos], kc.copy(), vc.copy(), q, k, v)


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


@pytest.mark.parametrize("B,H,HK,ctx", [(3, 16, 2, 700), (2, 64, 8, 2000), (1, 8, 8, 1)])
def test_gather_one_rank_matches_decode_and_oracle(B, H, HK, ctx):
    D = 128
    cu, kc, vc = _handle_with_cache(B, H, HK, D, ctx, 300 + ctx)
    ref_cu, _, _ = _handle_with_cache(B, H, HK, D, ctx, 300 + ctx)
    x = PeerExchange(0, 1, decode_xchg_bytes(SHARD_HEADS, 1, B, H, D), 0)
    out = torch.empty((B, H, D), device=DEV)
    for step, pos in enumerate((ctx, ctx + 1)):                 # two calls in a row
        q, k, v = (normal(310 + step, s, 3) for s in ((B, H, D), (B, HK, D), (B, HK, D)))
        cu.decode_gather_dev(x, 0, B, pos, _dev(q), _dev(k), _dev(v), out)
        want = torch.empty((B, H, D), device=DEV)
        ref_cu.decode_batch_dev(0, B, pos, _dev(q), _dev(k), _dev(v), want)
        cu.sync()
        x.sync()
        assert torch.equal(out, want), f"step {step}: fused gather differs from the decode"
        if step == 0:
            assert_rel(out.cpu().numpy(), _oracle(H, HK, D, pos, kc, vc, q, k, v), what="gather vs oracle")
    cu.close()
    ref_cu.close()
    x.close()


def test_gather_graph_replays_stay_correct():
    B, H, HK, D, ctx = 2, 32, 8, 128, 1500
    cu, _, _ = _handle_with_cache(B, H, HK, D, ctx, 41)
    ref_cu, _, _ = _handle_with_cache(B, H, HK, D, ctx, 41)
    x = PeerExchange(0, 1, decode_xchg_bytes(SHARD_HEADS, 1, B, H, D), 0)
    out = torch.empty((B, H, D), device=DEV)
    q, k, v = (_dev(normal(42, s, 1)) for s in ((B, H, D), (B, HK, D), (B, HK, D)))
    want = torch.empty((B, H, D), device=DEV)
    ref_cu.decode_batch_dev(0, B, ctx, q, k, v, want)
    st = torch.cuda.Stream(device=DEV)
    with torch.cuda.stream(st):
        cu.decode_gather_dev(x, 0, B, ctx, q, k, v, out, st)                # warm-up outside capture
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            cu.decode_gather_dev(x, 0, B, ctx, q, k, v, out, torch.cuda.current_stream())
    for rep in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"replay {rep}"
    x.sync()
    del g
    cu.close()
    ref_cu.close()
    x.close()


@pytest.mark.parametrize("B,H,HK,ctx,n_local", [(1, 32, 8, 3000, 3000), (2, 16, 4, 500, 500), (1, 8, 2, 0, 0)])
def test_seqshard_one_rank_matches_decode_and_oracle(B, H, HK, ctx, n_local):
    D = 128
    cu, kc, vc = _handle_with_cache(B, H, HK, D, ctx, 500 + ctx)
    ref_cu, _, _ = _handle_with_cache(B, H, HK, D, ctx, 500 + ctx)
    x = PeerExchange(0, 1, decode_xchg_bytes(SHARD_SEQ, 1, B, H, D), 0)
    out = torch.empty((B, H, D), device=DEV)
    want = torch.empty((B, H, D), device=DEV)
    for step, pos in enumerate((ctx, ctx + 1)):
        q, k, v = (normal(510 + step, s, 3) for s in ((B, H, D), (B, HK, D), (B, HK, D)))
        cu.decode_seqshard_dev(x, 0, B, pos, pos, True, _dev(q), _dev(k), _dev(v), out)
        ref_cu.decode_batch_dev(0, B, pos, _dev(q), _dev(k), _dev(v), want)
        cu.sync()
        x.sync()
        assert_rel(out.cpu().numpy(), want.cpu().numpy(), tol=1e-5, what=f"seqshard vs decode, step {step}")
        if step == 0:
            ref = _oracle(H, HK, D, pos, kc, vc, q, k, v)
            assert_rel(out.cpu().numpy(), ref, what="seqshard vs oracle")
    cu.close()
    ref_cu.close()
    x.close()


def test_absent_peer_times_out_breaks_the_exchange_and_leaves_the_gpu_usable():
    B, H, HK, D, ctx = 2, 16, 4, 128, 300
    cu, kc, vc = _handle_with_cache(B, H, HK, D, ctx, 61)
    nb = decode_xchg_bytes(SHARD_HEADS, 2, B, H, D)
    x0, x1 = PeerExchange(0, 2, nb, 0), PeerExchange(1, 2, nb, 0)
    x0.attach(1, x1)                        # rank 1 exists but never makes the call
    x0.set_wait(20_000_000)                 # 20 ms
    q, k, v = (normal(62, s, 1) for s in ((B, H, D), (B, HK, D), (B, HK, D)))
    # This handle plays rank 0 of a KV-head shard of 2 x H heads.
    out = torch.empty((B, 2 * H, D), device=DEV)
    cu.decode_gather_dev(x0, 0, B, ctx, _dev(q), _dev(k), _dev(v), out)
    cu.sync()                               # the decode itself is fine
    with pytest.raises(PickleError) as e:
        x0.sync()
    assert e.value.code == -9
    with pytest.raises(PickleError) as e:   # broken: the ranks' counters no longer agree
        cu.decode_gather_dev(x0, 0, B, ctx, _dev(q), _dev(k), _dev(v), out)
    assert e.value.code == -9
    # The unfused exchange gives up the same way.
    y0, y1 = PeerExchange(0, 2, nb, 0), PeerExchange(1, 2, nb, 0)
    y0.attach(1, y1)
    y0.set_wait(20_000_000)
    src = torch.zeros((B, H, D), device=DEV)
    row = B * H * D * 4
    y0.put(src, 1, row, row, 0, row)
    with pytest.raises(PickleError):
        y0.sync()
    with pytest.raises(PickleError):
        y0.put(src, 1, row, row, 0, row)
    # The GPU still decodes correctly.
    ao = torch.empty((B, H, D), device=DEV)
    cu.decode_batch_dev(0, B, ctx, _dev(q), _dev(k), _dev(v), ao)
    cu.sync()
    assert_rel(ao.cpu().numpy(), _oracle(H, HK, D, ctx, kc, vc, q, k, v), what="decode after the timeouts")
    for o in (x0, x1, y0, y1):
        o.close()
    cu.close()
