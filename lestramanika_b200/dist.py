"""Multi-GPU decode inside one box: one process per GPU, NCCL over NVLink.

Two sharding strategies for pickle's decode attention (the reference runs on
one host with OpenMP over heads only, src/pickle_fast.c:1960):

* KV-head-group sharding (HeadShardedDecode). Rank r owns KV heads
  [r*HK/N, (r+1)*HK/N) and their query heads (kv_head = h*HK/H,
  src/pickle_fast.c:1963, keeps every query head on the rank of its KV
  head), i.e. 1/N of the cache. Each rank decodes its heads; the head
  outputs [B][H/N][D] are all-gathered and laid out as [B][H][D].
* Sequence-chunk sharding (SeqShardedDecode). Rank r owns cache positions
  [r*S/N, (r+1)*S/N) of every head; the last rank appends the new token.
  Each rank computes the unnormalised triple (m, l, acc) of its chunk; the
  triples are all-gathered and merged by log-sum-exp.

The per-rank compute is a callable so the same orchestration runs with the
B200 kernels (device tensors) and, in the CPU tests, with a CPU computation
over gloo. On GPUs the exchange step is an NCCL all-gather or the library's
NVLink peer exchange (open_exchange): each rank stores its rows straight
into every rank's receive buffer at their final place, so the head slices
need no relayout. The exchange is either its own launch
(pickle_cuda_xchg_put_dev) or fused into the decode's split-merge launch
(pickle_cuda_decode_gather_dev, pickle_cuda_decode_seqshard_dev; the
benchmarks below). All ranks take the same collective steps in the same
order; process groups are created with a short timeout so a rank that
stops participating turns into an error on the others instead of a hang.
"""
import datetime
import os

from .workloads import head_shard, seq_shard


def init_group(backend, rank, world, timeout_s=60, device=None):
    """Join the default process group with a bounded collective timeout."""
    import torch
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = torch.device("cuda", device)
    dist.init_process_group(backend, rank=rank, world_size=world, **kw)


def open_exchange(rank, world, buf_bytes, device):
    """Create this rank's PeerExchange and open every other rank's receive
    region (the 64-byte CUDA IPC handles are all-gathered over the default
    process group)."""
    import torch
    import torch.distributed as dist
    from .api import IPC_HANDLE_BYTES, PeerExchange
    x = PeerExchange(rank, world, buf_bytes, device)
    dev = torch.device("cuda", device)
    mine = torch.frombuffer(bytearray(x.handle()), dtype=torch.uint8).to(dev)
    allh = torch.empty(world * IPC_HANDLE_BYTES, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(allh, mine)
    allh = allh.cpu().numpy().tobytes()
    for p in range(world):
        if p != rank:
            x.open(p, allh[p * IPC_HANDLE_BYTES:(p + 1) * IPC_HANDLE_BYTES])
    dist.barrier()
    return x


def merge_triples(m, l, acc):
    """Log-sum-exp merge of gathered partials (torch, any device).

    m, l: [N][rows]; acc: [N][rows][D] ->  out [rows][D] =
    sum_i e^(m_i - M) acc_i / sum_i e^(m_i - M) l_i,  M = max_i m_i.
    (The B200 path runs the same formula in lse_merge_kernel.)
    """
    import torch
    M = m.max(dim=0).values
    w = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), torch.exp(m - M))
    L = (w * l).sum(dim=0)
    L = torch.where(L == 0, torch.ones_like(L), L)
    return (w.unsqueeze(-1) * acc).sum(dim=0) / L.unsqueeze(-1)


class HeadShardedDecode:
    """KV-head-group sharded decode step for one rank.

    compute(q, k, v, out) fills out [B][H/N][D] for this rank's heads;
    step() returns the all-gathered [B][H][D]. With exchange (a
    PeerExchange of B*H*D*4 bytes) the rows go straight into every rank's
    [B][H][D] receive buffer; without it, NCCL all-gather and a relayout.
    """

    def __init__(self, B, H, HK, D, rank, world, compute, device=None, dtype=None, exchange=None):
        import torch
        (self.h0, self.h1), (self.k0, self.k1) = head_shard_dims(H, HK, world, rank)
        self.B, self.H, self.HK, self.D, self.world = B, H, HK, D, world
        self.compute = compute
        dev = torch.device("cpu") if device is None else torch.device("cuda", device)
        dtype = dtype or torch.float32
        self.local = torch.empty((B, self.h1 - self.h0, D), device=dev, dtype=dtype)
        # Flat [N*B][H/N][D]: all_gather_into_tensor concatenates along dim 0.
        self.gathered = torch.empty((world * B, self.h1 - self.h0, D), device=dev, dtype=dtype)
        self.out = torch.empty((B, H, D), device=dev, dtype=dtype)
        self.exchange = exchange
        if exchange is not None:
            self.out = exchange.buffer((B, H, D))

    def slice_inputs(self, q, k, v):
        """This rank's share of full [B][H][D] q and [B][HK][D] k/v."""
        return (q[:, self.h0:self.h1].contiguous(), k[:, self.k0:self.k1].contiguous(),
                v[:, self.k0:self.k1].contiguous())

    def step(self, q_local, k_local, v_local):
        import torch.distributed as dist
        self.compute(q_local, k_local, v_local, self.local)
        if self.exchange is not None:
            import torch
            row = (self.h1 - self.h0) * self.D * 4
            self.exchange.put(self.local, self.B, row, row, self.h0 * self.D * 4, self.H * self.D * 4,
                              torch.cuda.current_stream(self.local.device))
            return self.out
        dist.all_gather_into_tensor(self.gathered, self.local)
        # [N][B][H/N][D] -> [B][N][H/N][D] = [B][H][D]
        g = self.gathered.view(self.world, self.B, self.h1 - self.h0, self.D)
        self.out.view(self.B, self.world, self.h1 - self.h0, self.D).copy_(g.transpose(0, 1))
        return self.out


def head_shard_dims(H, HK, world, rank):
    if HK % world or H % world:
        raise ValueError(f"{H} query / {HK} KV heads do not split {world} ways")
    hk, h = HK // world, H // world
    return (rank * h, (rank + 1) * h), (rank * hk, (rank + 1) * hk)


class SeqShardedDecode:
    """Sequence-chunk sharded decode step for one rank.

    Each rank's partial triple lives in one packed buffer
    part = [acc (rows x D) | m (rows) | l (rows)], rows = B*H, so a step is
    one all-gather. compute(q, k, v, m, l, acc) fills this rank's views;
    merge(parts, part_stride, out) merges the gathered [N] parts (default:
    merge_triples on views). step() returns out [B][H][D]. With exchange (a
    PeerExchange of N*part bytes) the parts land in its receive buffer.
    """

    def __init__(self, B, H, D, ctx, rank, world, compute, merge=None, device=None, exchange=None):
        import torch
        self.p0, self.p1 = seq_shard(ctx, world, rank)
        self.append = rank == world - 1
        self.B, self.H, self.D, self.world = B, H, D, world
        self.compute = compute
        self.merge = merge
        dev = torch.device("cpu") if device is None else torch.device("cuda", device)
        self.rows = rows = B * H
        self.stride = (rows * (D + 2) + 3) // 4 * 4          # parts start on 16-byte boundaries
        self.part = torch.empty(self.stride, device=dev)
        self.acc = self.part[:rows * D].view(rows, D)
        self.m = self.part[rows * D:rows * (D + 1)]
        self.l = self.part[rows * (D + 1):]
        self.parts = torch.empty(world * self.stride, device=dev)
        self.out = torch.empty((B, H, D), device=dev)
        self.rank = rank
        self.exchange = exchange
        if exchange is not None:
            self.parts = exchange.buffer((world * self.stride,))

    @property
    def n_local(self):
        return self.p1 - self.p0

    def step(self, q, k, v):
        import torch.distributed as dist
        self.compute(q, k, v, self.m, self.l, self.acc)
        if self.exchange is not None:
            import torch
            nb = self.stride * 4
            self.exchange.put(self.part, 1, nb, nb, self.rank * nb, nb, torch.cuda.current_stream(self.part.device))
        else:
            dist.all_gather_into_tensor(self.parts, self.part)
        if self.merge is not None:
            self.merge(self.parts, self.stride, self.out)
        else:
            rows, D = self.rows, self.D
            p = self.parts.view(self.world, self.stride)
            self.out.view(-1, D).copy_(merge_triples(p[:, rows * D:rows * (D + 1)], p[:, rows * (D + 1):],
                                                     p[:, :rows * D].reshape(self.world, rows, D)))
        return self.out


# ---------------------------------------------------------------------------
# B200 benchmarks of the two strategies (called by bench.py under torchrun)
# ---------------------------------------------------------------------------

def _max_over_ranks(ms, device):
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device=torch.device("cuda", device))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(fn, steps, warmup, device, graph=False):
    """Device time per step (ms), max over ranks. graph=True captures the
    `steps` calls (collectives included) in one CUDA graph and replays it
    between the events, as a serving loop replays its decode step; the
    graph is released before returning."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(steps):
                fn()
        g.replay()
        torch.cuda.synchronize(device)
    dist.barrier()
    torch.cuda.synchronize(device)
    st = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    if g is not None:
        g.replay()
    else:
        for _ in range(steps):
            fn()
    e1.record(st)
    torch.cuda.synchronize(device)
    del g
    dist.barrier()
    return _max_over_ranks(e0.elapsed_time(e1) / steps, device)


def _fill_rows(kt, vt, rows, g, B):
    """Seeded N(0, 1) cache rows [0, rows) of every sequence and KV head of a
    [B][heads][max_seq][D] view, drawn contiguously (so the values depend
    only on the generator, not on the view's strides)."""
    import torch
    for b in range(B):
        shape = (kt.shape[1], rows, kt.shape[3])
        kt[b, :, :rows].copy_(torch.randn(shape, generator=g, device=kt.device))
        vt[b, :, :rows].copy_(torch.randn(shape, generator=g, device=vt.device))


def head_shard_data(w, world, rank, kt, vt):
    """Rank `rank`'s KV-head shard of workload w: its cache rows into kt/vt
    ([B][HK/N][>= ctx][D] views) and its q [B][H/N][D], k, v [B][HK/N][D]."""
    import torch
    (h0, h1), (k0, k1) = head_shard(w, world, rank)
    g = torch.Generator(device=kt.device)
    g.manual_seed(1000 + rank)
    _fill_rows(kt, vt, w.ctx, g, w.B)
    q = torch.randn((w.B, h1 - h0, w.D), generator=g, device=kt.device)
    k = torch.randn((w.B, k1 - k0, w.D), generator=g, device=kt.device)
    v = torch.randn((w.B, k1 - k0, w.D), generator=g, device=kt.device)
    return q, k, v


def seq_shard_data(w, world, rank, kt, vt):
    """Rank `rank`'s cache chunk of workload w into kt/vt ([B][HK][>= n_local][D]
    views); q/k/v are the same on every rank."""
    import torch
    p0, p1 = seq_shard(w.ctx, world, rank)
    g = torch.Generator(device=kt.device)
    g.manual_seed(2000 + rank)
    _fill_rows(kt, vt, p1 - p0, g, w.B)
    g.manual_seed(7)
    q = torch.randn((w.B, w.H, w.D), generator=g, device=kt.device)
    k = torch.randn((w.B, w.HK, w.D), generator=g, device=kt.device)
    v = torch.randn((w.B, w.HK, w.D), generator=g, device=kt.device)
    return q, k, v


def _one_gpu_reference(w, world, device, steps, warmup, kind):
    """Rank 0 only: the whole workload on this one GPU, its cache assembled
    from every rank's seeded shard - the unsharded decode's output (the
    parity reference of the sharded run) and its device time per step."""
    import torch
    from .api import PickleCuda
    cu = PickleCuda(1, w.H, w.HK, w.D, w.ctx + 1, rope_theta=w.theta, n_seqs=w.B, device=device)
    kt, vt = cu.kv_tensors(0)
    dev = torch.device("cuda", device)
    q = torch.empty((w.B, w.H, w.D), device=dev)
    k = torch.empty((w.B, w.HK, w.D), device=dev)
    v = torch.empty((w.B, w.HK, w.D), device=dev)
    for r in range(world):
        if kind == "head":
            (h0, h1), (k0, k1) = head_shard(w, world, r)
            qr, kr, vr = head_shard_data(w, world, r, kt[:, k0:k1], vt[:, k0:k1])
            q[:, h0:h1], k[:, k0:k1], v[:, k0:k1] = qr, kr, vr
        else:
            p0, p1 = seq_shard(w.ctx, world, r)
            q, k, v = seq_shard_data(w, world, r, kt[:, :, p0:p1], vt[:, :, p0:p1])
    out = torch.empty((w.B, w.H, w.D), device=dev)
    st = torch.cuda.current_stream(device)
    for _ in range(warmup):
        cu.decode_batch_dev(0, w.B, w.ctx, q, k, v, out, st)
    cu.sync(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(steps):
            cu.decode_batch_dev(0, w.B, w.ctx, q, k, v, out, torch.cuda.current_stream(device))
    g.replay()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    del g
    cu.decode_batch_dev(0, w.B, w.ctx, q, k, v, out, st)
    cu.sync(st)
    cu.close()
    return out, ms


def _rel_err(got, ref):
    return float(((got - ref).abs().max() / ref.abs().max()).item())


def bench_head_sharded(w, rank, world, device, steps, warmup):
    """KV-head shard of w on `world` ranks: the decode with the head
    exchange fused into its merge launch (pickle_cuda_decode_gather_dev) is
    the headline; timed beside it: the same decode with an NCCL all-gather,
    the per-GPU decode kernel alone, and the end-to-end step from host
    buffers. Rank 0 checks the gathered output against the whole problem
    decoded on one GPU and times that too (the 1-GPU point of the strong
    scaling)."""
    import torch
    import torch.distributed as dist
    from .api import SHARD_HEADS, PickleCuda, decode_xchg_bytes
    (h0, h1), (k0, k1) = head_shard(w, world, rank)
    H, HK = h1 - h0, k1 - k0
    cu = PickleCuda(1, H, HK, w.D, w.ctx + 1, rope_theta=w.theta, n_seqs=w.B, device=device)
    kt, vt = cu.kv_tensors(0)
    q, k, v = head_shard_data(w, world, rank, kt, vt)
    st = torch.cuda.current_stream(device)

    def compute(qq, kk, vv, out):
        cu.decode_batch_dev(0, w.B, w.ctx, qq, kk, vv, out, torch.cuda.current_stream(device))

    hs_nccl = HeadShardedDecode(w.B, w.H, w.HK, w.D, rank, world, compute, device=device)
    nccl_ms = _timed(lambda: hs_nccl.step(q, k, v), steps, warmup, device, graph=True)
    x = open_exchange(rank, world, decode_xchg_bytes(SHARD_HEADS, world, w.B, H, w.D), device)
    out = torch.empty((w.B, w.H, w.D), device=torch.device("cuda", device))

    def fused():
        cu.decode_gather_dev(x, 0, w.B, w.ctx, q, k, v, out, torch.cuda.current_stream(device))

    ms = _timed(fused, steps, warmup, device, graph=True)
    local = torch.empty((w.B, H, w.D), device=torch.device("cuda", device))
    kernel_ms = _timed(lambda: compute(q, k, v, local), steps, warmup, device, graph=True)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(out.shape).pin_memory()

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        k.copy_(hk, non_blocking=True)
        v.copy_(hv, non_blocking=True)
        fused()
        hout.copy_(out, non_blocking=True)

    e2e_ms = _timed(e2e_step, steps, warmup, device)
    fused()
    cu.sync(st)
    x.sync(st)
    got = out.clone()
    splits = cu.decode_plan(w.B, w.ctx)[0]
    cu.close()
    dist.barrier()
    ref = None
    if rank == 0:
        ref_out, one_ms = _one_gpu_reference(w, world, device, steps, warmup, "head")
        ref = {"max_rel_err_vs_one_gpu": _rel_err(got, ref_out), "one_gpu_ms": one_ms}
    dist.barrier()
    x.close()
    per_gpu = w.kv_bytes / world
    return {"ms": ms, "kernel_ms": kernel_ms, "kernel_GBps_per_gpu": per_gpu / (kernel_ms * 1e-3) / 1e9,
            "launches_per_step": 2, "splits": splits, "nccl_all_gather_ms": nccl_ms, "one_gpu": ref,
            "e2e": {"value": w.kv_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": sum(t.numel() * 4 for t in (hq, hk, hv)),
                    "d2h_bytes_per_step": hout.numel() * 4, "ms_per_step": e2e_ms}}


def bench_seq_sharded(w, rank, world, device, steps, warmup):
    """Sequence-chunk shard of w on `world` ranks: the partial decode with
    the triple exchange and log-sum-exp merge fused into its merge launch
    (pickle_cuda_decode_seqshard_dev); the NCCL all-gather + merge variant
    timed beside it; rank 0 checks the output against the whole problem on
    one GPU and times that."""
    import torch
    import torch.distributed as dist
    from .api import SHARD_SEQ, PickleCuda, decode_xchg_bytes, lse_merge_packed_dev
    p0, p1 = seq_shard(w.ctx, world, rank)
    n_local = p1 - p0
    append = rank == world - 1
    cu = PickleCuda(1, w.H, w.HK, w.D, n_local + 1, rope_theta=w.theta, n_seqs=w.B, rope_len=w.ctx + 1,
                    device=device)
    kt, vt = cu.kv_tensors(0)
    q, k, v = seq_shard_data(w, world, rank, kt, vt)
    st = torch.cuda.current_stream(device)

    def compute(qq, kk, vv, m, l, acc):
        cu.decode_partial_dev(0, w.B, w.ctx, n_local, append, qq, kk, vv, m, l, acc,
                              torch.cuda.current_stream(device))

    def merge(parts, stride, out):
        lse_merge_packed_dev(world, w.B * w.H, w.D, parts, stride, out, torch.cuda.current_stream(device))

    ss_nccl = SeqShardedDecode(w.B, w.H, w.D, w.ctx, rank, world, compute, merge=merge, device=device)
    nccl_ms = _timed(lambda: ss_nccl.step(q, k, v), steps, warmup, device, graph=True)
    x = open_exchange(rank, world, decode_xchg_bytes(SHARD_SEQ, world, w.B, w.H, w.D), device)
    out = torch.empty((w.B, w.H, w.D), device=torch.device("cuda", device))

    def fused():
        cu.decode_seqshard_dev(x, 0, w.B, w.ctx, n_local, append, q, k, v, out, torch.cuda.current_stream(device))

    ms = _timed(fused, steps, warmup, device, graph=True)
    m_, l_ = torch.empty(w.B * w.H, device=out.device), torch.empty(w.B * w.H, device=out.device)
    acc_ = torch.empty((w.B * w.H, w.D), device=out.device)
    kernel_ms = _timed(lambda: compute(q, k, v, m_, l_, acc_), steps, warmup, device, graph=True)
    fused()
    cu.sync(st)
    x.sync(st)
    got = out.clone()
    cu.close()
    dist.barrier()
    ref = None
    if rank == 0:
        ref_out, one_ms = _one_gpu_reference(w, world, device, steps, warmup, "seq")
        ref = {"max_rel_err_vs_one_gpu": _rel_err(got, ref_out), "one_gpu_ms": one_ms}
    dist.barrier()
    x.close()
    per_gpu = w.kv_bytes / world
    return {"ms": ms, "kernel_ms": kernel_ms, "kernel_GBps_per_gpu": per_gpu / (kernel_ms * 1e-3) / 1e9,
            "nccl_all_gather_ms": nccl_ms, "one_gpu": ref}
