"""Worker of tests/test_multigpu_xchg_gpu.py, one process per GPU under
torchrun: both sharded decodes through the NVLink peer exchange - the
separate put launch and the exchange fused into the merge launch
(pickle_cuda_decode_gather_dev / pickle_cuda_decode_seqshard_dev) - must
give the NCCL all-gather path's outputs (exactly for the head shard, within
1e-5 relative for the log-sum-exp merge), on several steps in a row and from
a replayed CUDA graph."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from lestramanika_b200 import PickleCuda, lse_merge_packed_dev  # noqa: E402
from lestramanika_b200.api import SHARD_HEADS, SHARD_SEQ, decode_xchg_bytes  # noqa: E402
from lestramanika_b200.dist import HeadShardedDecode, SeqShardedDecode, init_group, open_exchange  # noqa: E402
from lestramanika_b200.workloads import Decode, head_shard, seq_shard  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev_i = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(dev_i)
    init_group("nccl", rank, world, timeout_s=60, device=dev_i)
    dev = torch.device("cuda", dev_i)
    bad = []

    # KV-head shard
    w = Decode("t", 3, 16, 8, 128, 700, 500000.0)
    (h0, h1), (k0, k1) = head_shard(w, world, rank)
    cu = PickleCuda(1, h1 - h0, k1 - k0, w.D, w.ctx + 1, rope_theta=w.theta, n_seqs=w.B, device=dev_i)
    kt, vt = cu.kv_tensors(0)
    g = torch.Generator(device=dev)
    g.manual_seed(100 + rank)
    kt.normal_(generator=g)
    vt.normal_(generator=g)

    def compute(qq, kk, vv, out):
        cu.decode_batch_dev(0, w.B, w.ctx, qq, kk, vv, out, torch.cuda.current_stream(dev_i))

    x = open_exchange(rank, world, w.B * w.H * w.D * 4, dev_i)
    xf = open_exchange(rank, world, decode_xchg_bytes(SHARD_HEADS, world, w.B, h1 - h0, w.D), dev_i)
    fused_out = torch.empty((w.B, w.H, w.D), device=dev)
    a = HeadShardedDecode(w.B, w.H, w.HK, w.D, rank, world, compute, device=dev_i)
    b = HeadShardedDecode(w.B, w.H, w.HK, w.D, rank, world, compute, device=dev_i, exchange=x)

    def fused_step(qq, kk, vv):
        cu.decode_gather_dev(xf, 0, w.B, w.ctx, qq, kk, vv, fused_out, torch.cuda.current_stream(dev_i))

    for step in range(3):
        q = torch.randn((w.B, h1 - h0, w.D), generator=g, device=dev)
        k = torch.randn((w.B, k1 - k0, w.D), generator=g, device=dev)
        v = torch.randn((w.B, k1 - k0, w.D), generator=g, device=dev)
        want = a.step(q, k, v).clone()
        got = b.step(q, k, v).clone()
        if not torch.equal(got, want):
            bad.append(f"head shard step {step}")
        fused_step(q, k, v)
        torch.cuda.synchronize()
        if not torch.equal(fused_out, want):
            bad.append(f"fused head shard step {step}")
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        b.step(q, k, v)
        fused_step(q, k, v)
    for rep in range(2):
        fused_out.zero_()
        gr.replay()
        torch.cuda.synchronize()
        if not torch.equal(b.out, want):
            bad.append(f"head shard replay {rep}")
        if not torch.equal(fused_out, want):
            bad.append(f"fused head shard replay {rep}")
    del gr
    x.sync()
    xf.sync()
    cu.close()

    # sequence-chunk shard
    w = Decode("t", 2, 16, 8, 128, 1500, 500000.0)
    p0, p1 = seq_shard(w.ctx, world, rank)
    n_local = p1 - p0
    append = rank == world - 1
    cu = PickleCuda(1, w.H, w.HK, w.D, n_local + 1, rope_theta=w.theta, n_seqs=w.B, rope_len=w.ctx + 1,
                    device=dev_i)
    kt, vt = cu.kv_tensors(0)
    kt.normal_(generator=g)
    vt.normal_(generator=g)

    def pcompute(qq, kk, vv, m, l, acc):
        cu.decode_partial_dev(0, w.B, w.ctx, n_local, append, qq, kk, vv, m, l, acc,
                              torch.cuda.current_stream(dev_i))

    def merge(parts, stride, out):
        lse_merge_packed_dev(world, w.B * w.H, w.D, parts, stride, out, torch.cuda.current_stream(dev_i))

    sa = SeqShardedDecode(w.B, w.H, w.D, w.ctx, rank, world, pcompute, merge=merge, device=dev_i)
    x2 = open_exchange(rank, world, world * sa.stride * 4, dev_i)
    sb = SeqShardedDecode(w.B, w.H, w.D, w.ctx, rank, world, pcompute, merge=merge, device=dev_i, exchange=x2)
    xs = open_exchange(rank, world, decode_xchg_bytes(SHARD_SEQ, world, w.B, w.H, w.D), dev_i)
    sout = torch.empty((w.B, w.H, w.D), device=dev)

    def fused_seq(qq, kk, vv):
        cu.decode_seqshard_dev(xs, 0, w.B, w.ctx, n_local, append, qq, kk, vv, sout,
                               torch.cuda.current_stream(dev_i))

    def close(a_, b_):
        err = ((a_ - b_).abs().max() / b_.abs().max()).item()
        return err <= 1e-5

    gq = torch.Generator(device=dev)
    gq.manual_seed(7)
    for step in range(3):
        q = torch.randn((w.B, w.H, w.D), generator=gq, device=dev)
        k = torch.randn((w.B, w.HK, w.D), generator=gq, device=dev)
        v = torch.randn((w.B, w.HK, w.D), generator=gq, device=dev)
        want = sa.step(q, k, v).clone()
        got = sb.step(q, k, v).clone()
        if not torch.equal(got, want):
            bad.append(f"seq shard step {step}")
        fused_seq(q, k, v)
        torch.cuda.synchronize()
        if not close(sout, want):
            bad.append(f"fused seq shard step {step}")
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        fused_seq(q, k, v)
    for rep in range(3):
        sout.zero_()
        gr.replay()
        torch.cuda.synchronize()
        if not close(sout, want):
            bad.append(f"fused seq shard replay {rep}")
    del gr
    x2.sync()
    xs.sync()
    cu.close()
    torch.cuda.synchronize()
    dist.barrier()
    x.close()
    xf.close()
    x2.close()
    xs.close()
    dist.destroy_process_group()
    if bad:
        print(f"rank {rank}: MISMATCH {bad}", flush=True)
        sys.exit(1)
    print(f"rank {rank}: ok", flush=True)


if __name__ == "__main__":
    main()
