"""Multi-rank orchestration on CPU (gloo, world_size 2): the sharding plans,
the all-gather layouts, the log-sum-exp merge and failure handling, with the
per-rank attention computed on the CPU (oracle). No GPU."""
import os
import socket
import sys
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from lestramanika_b200.dist import init_group
    init_group("gloo", rank, world, timeout_s=timeout_s)


def _case(B, H, HK, D, ctx, seed):
    rng = np.random.Generator(np.random.Philox(seed))
    kc = np.zeros((B, ctx + 1, HK, D), np.float32)
    vc = np.zeros((B, ctx + 1, HK, D), np.float32)
    kc[:, :ctx] = rng.standard_normal((B, ctx, HK, D), dtype=np.float32)
    vc[:, :ctx] = rng.standard_normal((B, ctx, HK, D), dtype=np.float32)
    q = rng.standard_normal((B, H, D), dtype=np.float32)
    k = rng.standard_normal((B, HK, D), dtype=np.float32)
    v = rng.standard_normal((B, HK, D), dtype=np.float32)
    return kc, vc, q, k, v


def _head_rank(rank, world, port, out_dir):
    _init(rank, world, port)
    import torch.distributed as dist

    import oracle
    from lestramanika_b200.dist import HeadShardedDecode
    B, H, HK, D, ctx = 2, 8, 4, 64, 50
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 3)
    _, s, c = oracle.rope_tables(10000.0, D, ctx + 1)

    def compute(qq, kk, vv, out):
        k0, k1 = hs.k0, hs.k1
        kcs = np.ascontiguousarray(kc[:, :, k0:k1])
        vcs = np.ascontiguousarray(vc[:, :, k0:k1])
        ao = oracle.decode_batch(hs.h1 - hs.h0, k1 - k0, D, ctx, s[ctx], c[ctx], kcs, vcs,
                                 qq.numpy(), kk.numpy(), vv.numpy())
        out.copy_(torch.from_numpy(ao))

    hs = HeadShardedDecode(B, H, HK, D, rank, world, compute)
    ql, kl, vl = hs.slice_inputs(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v))
    out = hs.step(ql, kl, vl)
    np.save(os.path.join(out_dir, f"head{rank}.npy"), out.numpy())
    dist.destroy_process_group()


def _seq_rank(rank, world, port, out_dir):
    _init(rank, world, port)
    import torch.distributed as dist

    import oracle
    from lestramanika_b200.dist import SeqShardedDecode
    B, H, HK, D, ctx = 2, 8, 2, 64, 77
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 4)
    _, s, c = oracle.rope_tables(10000.0, D, ctx + 1)
    G = H // HK

    def compute(qq, kk, vv, m, l, acc):
        # Partial triple over this rank's rows [p0, p1) (+ the new row on the last rank), float64.
        qr = oracle.rope_apply(qq.numpy(), D, s[ctx], c[ctx]).astype(np.float64)
        kr = oracle.rope_apply(kk.numpy(), D, s[ctx], c[ctx]).astype(np.float64)
        rows_k = kc[:, ss.p0:ss.p1].astype(np.float64)
        rows_v = vc[:, ss.p0:ss.p1].astype(np.float64)
        if ss.append:
            rows_k = np.concatenate([rows_k, kr[:, None]], axis=1)
            rows_v = np.concatenate([rows_v, vv.numpy()[:, None].astype(np.float64)], axis=1)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        mm, ll, aa = [], [], []
        for b in range(B):
            for h in range(H):
                sc = rows_k[b, :, h // G] @ qr[b, h] * scale
                mx = sc.max()
                e = np.exp(sc - mx)
                mm.append(mx)
                ll.append(e.sum())
                aa.append(e @ rows_v[b, :, h // G])
        m.copy_(torch.tensor(mm))
        l.copy_(torch.tensor(ll))
        acc.copy_(torch.tensor(np.array(aa)))

    ss = SeqShardedDecode(B, H, D, ctx, rank, world, compute)
    out = ss.step(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v))
    np.save(os.path.join(out_dir, f"seq{rank}.npy"), out.numpy())
    dist.destroy_process_group()


def _silent_rank(rank, world, port, out_dir):
    """Rank 1 leaves before the collective; rank 0 must get an error, not hang."""
    _init(rank, world, port, timeout_s=5)
    import torch.distributed as dist
    if rank == 1:
        dist.barrier()
        return                                   # never joins the all-gather
    dist.barrier()
    t0 = time.time()
    try:
        out = torch.empty(4)
        dist.all_gather_into_tensor(out, torch.ones(2))
        status = "completed"
    except Exception as exc:                     # gloo timeout / peer closed
        status = f"error:{type(exc).__name__}"
    with open(os.path.join(out_dir, "silent.txt"), "w") as f:
        f.write(f"{status} {time.time() - t0:.1f}")


def test_head_sharded_matches_full_attention(tmp_path):
    mp.spawn(_head_rank, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    import oracle
    B, H, HK, D, ctx = 2, 8, 4, 64, 50
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 3)
    _, s, c = oracle.rope_tables(10000.0, D, ctx + 1)
    ref = oracle.decode_batch(H, HK, D, ctx, s[ctx], c[ctx], kc, vc, q, k, v)
    for r in range(2):
        got = np.load(tmp_path / f"head{r}.npy")
        np.testing.assert_array_equal(got, ref)   # same oracle per head, gathered in order


def test_seq_sharded_lse_merge_matches_full_attention(tmp_path):
    mp.spawn(_seq_rank, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    import oracle
    B, H, HK, D, ctx = 2, 8, 2, 64, 77
    kc, vc, q, k, v = _case(B, H, HK, D, ctx, 4)
    _, s, c = oracle.rope_tables(10000.0, D, ctx + 1)
    ref = oracle.decode_batch(H, HK, D, ctx, s[ctx], c[ctx], kc, vc, q, k, v)
    for r in range(2):
        got = np.load(tmp_path / f"seq{r}.npy")
        assert np.max(np.abs(got - ref)) / np.max(np.abs(ref)) <= 1e-5


def test_peer_that_leaves_turns_into_an_error(tmp_path):
    mp.spawn(_silent_rank, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    status, secs = open(tmp_path / "silent.txt").read().split()
    assert status.startswith("error"), status
    assert float(secs) < 60


def test_shard_plans():
    from lestramanika_b200.dist import head_shard_dims, merge_triples
    from lestramanika_b200.workloads import C4, head_shard, seq_shard
    # every query head stays with its KV head (kv_head = h*HK/H)
    for world in (1, 2, 4, 8):
        for r in range(world):
            (h0, h1), (k0, k1) = head_shard(C4, world, r)
            assert all(k0 <= h * C4.HK // C4.H < k1 for h in range(h0, h1))
    with pytest.raises(ValueError):
        head_shard_dims(64, 8, 3, 0)
    # chunks tile [0, ctx) exactly
    for world in (1, 2, 4, 8):
        spans = [seq_shard(131072, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 131072
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    # merge of a single part is its normalisation; empty parts (m=-inf) drop out
    m = torch.tensor([[0.5, -float("inf")], [-float("inf"), 1.0]])
    l = torch.tensor([[2.0, 0.0], [0.0, 4.0]])
    acc = torch.tensor([[[2.0, 4.0], [0.0, 0.0]], [[0.0, 0.0], [8.0, 4.0]]])
    out = merge_triples(m, l, acc)
    assert torch.allclose(out, torch.tensor([[1.0, 2.0], [2.0, 1.0]]))
