"""The sharded decode paths on one GPU: each shard is its own handle, run in
turn, and the results are combined exactly as the multi-GPU code combines
them (head outputs concatenated; partial (m, l, acc) triples merged by
log-sum-exp), then compared with the whole-cache oracle."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import assert_rel, normal
from lestramanika_b200 import PickleCuda, lse_merge_dev, lse_merge_packed_dev
from lestramanika_b200.workloads import Decode, head_shard, seq_shard

pytestmark = pytest.mark.gpu


def _case(B, H, HK, D, ctx, seed):
    kc = np.zeros((B, ctx + 1, HK, D), np.float32)
    vc = np.zeros((B, ctx + 1, HK, D), np.float32)
    kc[:, :ctx] = normal(seed, (B, ctx, HK, D), 1)
    vc[:, :ctx] = normal(seed, (B, ctx, HK, D), 2)
    return kc, vc, normal(seed, (B, H, D), 3), normal(seed, (B, HK, D), 4), normal(seed, (B, HK, D), 5)


def _ref(B, H, HK, D, ctx, kc, vc, q, k, v, theta):
    _, s, c = oracle.rope_tables(theta, D, ctx + 1)
    return oracle.decode_batch(H, HK, D, ctx, s[ctx], c[ctx], kc.copy(), vc.copy(), q, k, v)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_shards_concatenate_to_full_attention(world):
    B, H, HK, D, ctx, theta = 3, 64, 8, 128, 700, 500000.0
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 40 + world)
    ref = _ref(B, H, HK, D, ctx, kc, vc, q, k, v, theta)
    dev = torch.device("cuda", 0)
    w = Decode("t", B, H, HK, D, ctx, theta)
    out = np.empty_like(ref)
    for r in range(world):
        (h0, h1), (k0, k1) = head_shard(w, world, r)
        cu = PickleCuda(1, h1 - h0, k1 - k0, D, ctx + 1, rope_theta=theta, n_seqs=B)
        for b in range(B):
            cu.kv_write(0, b, 0, kc[b, :ctx, k0:k1], vc[b, :ctx, k0:k1])
        qd = torch.from_numpy(np.ascontiguousarray(q[:, h0:h1])).to(dev)
        kd = torch.from_numpy(np.ascontiguousarray(k[:, k0:k1])).to(dev)
        vd = torch.from_numpy(np.ascontiguousarray(v[:, k0:k1])).to(dev)
        ao = torch.empty((B, h1 - h0, D), device=dev)
        cu.decode_batch_dev(0, B, ctx, qd, kd, vd, ao)
        cu.sync()
        out[:, h0:h1] = ao.cpu().numpy()
        cu.close()
    assert_rel(out, ref, what=f"kv-head shards x{world}")


@pytest.mark.parametrize("world,packed", [(2, True), (3, False), (8, True)])
def test_sequence_chunks_merge_to_full_attention(world, packed):
    B, H, HK, D, ctx, theta = 2, 32, 8, 128, 1000, 500000.0
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 50 + world)
    ref = _ref(B, H, HK, D, ctx, kc, vc, q, k, v, theta)
    dev = torch.device("cuda", 0)
    rows = B * H
    stride = rows * (D + 2)
    parts = torch.empty(world * stride, device=dev)
    m_all = torch.empty((world, rows), device=dev)
    l_all = torch.empty((world, rows), device=dev)
    acc_all = torch.empty((world, rows, D), device=dev)
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    for r in range(world):
        p0, p1 = seq_shard(ctx, world, r)
        n_local = p1 - p0
        append = r == world - 1
        cu = PickleCuda(1, H, HK, D, n_local + 1, rope_theta=theta, n_seqs=B, rope_len=ctx + 1)
        for b in range(B):
            cu.kv_write(0, b, 0, kc[b, p0:p1], vc[b, p0:p1])
        if packed:
            part = parts[r * stride:(r + 1) * stride]
            cu.decode_partial_dev(0, B, ctx, n_local, append, qd, kd, vd, part[rows * D:rows * (D + 1)],
                                  part[rows * (D + 1):], part[:rows * D])
        else:
            cu.decode_partial_dev(0, B, ctx, n_local, append, qd, kd, vd, m_all[r], l_all[r], acc_all[r])
        cu.sync()
        cu.close()
    out = torch.empty((B, H, D), device=dev)
    if packed:
        lse_merge_packed_dev(world, rows, D, parts, stride, out)
    else:
        lse_merge_dev(world, rows, D, m_all, l_all, acc_all, out)
    torch.cuda.synchronize()
    assert_rel(out.cpu().numpy(), ref, what=f"sequence chunks x{world} packed={packed}")


def test_peer_exchange_single_rank_places_rows_across_calls_and_graph_replays():
    """The NVLink exchange with one rank: a [B][H/2][D] head slice lands at
    its place in the [B][H][D] receive buffer, on consecutive calls (the
    device-side call counters advance) and when the call is replayed from a
    CUDA graph."""
    from lestramanika_b200.api import PeerExchange
    dev = torch.device("cuda", 0)
    B, H, D, h0 = 3, 8, 128, 4
    x = PeerExchange(0, 1, B * H * D * 4, 0)
    buf = x.buffer((B, H, D))
    row = (H // 2) * D * 4
    st = torch.cuda.current_stream()
    for call in range(2):
        src = torch.randn((B, H // 2, D), device=dev)
        x.put(src, B, row, row, h0 * D * 4, H * D * 4, st)
        x.sync(st)
        assert torch.equal(buf[:, h0:], src), f"call {call}"
    src = torch.zeros((B, H // 2, D), device=dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        x.put(src, B, row, row, h0 * D * 4, H * D * 4, torch.cuda.current_stream())
    for rep in range(2):
        src.copy_(torch.randn((B, H // 2, D), device=dev))
        g.replay()
        x.sync(st)
        assert torch.equal(buf[:, h0:], src), f"replay {rep}"
    del g
    x.close()


def test_peer_exchange_rejects_rows_outside_the_buffer():
    from lestramanika_b200 import PickleError
    from lestramanika_b200.api import PeerExchange
    x = PeerExchange(0, 1, 4096, 0)
    src = torch.zeros(2048, device=torch.device("cuda", 0))
    with pytest.raises(PickleError) as e:
        x.put(src, 2, 4096, 4096, 0, 4096)
    assert e.value.code == -7
    x.close()
