"""The synthetic workloads of the benchmark and the multi-GPU runs.

Shapes are the configurations the reference's attention block is measured
on (Llama-3-8B / Llama-2-7B / Llama-3-70B shaped), with seeded N(0, 1)
inputs generated on the device (cache) or host (new q/k/v).
Algorithmic work per step:
  decode: bytes = B * HK * (ctx + 1) * D * 4 * 2   (one read of K and V rows)
  prefill: flops = 4 * B * H * D * T * (T + 1) / 2 (QK^T and PV over causal pairs)
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Decode:
    name: str
    B: int
    H: int
    HK: int
    D: int
    ctx: int
    theta: float

    @property
    def kv_bytes(self):
        return self.B * self.HK * (self.ctx + 1) * self.D * 4 * 2

    @property
    def G(self):
        return self.H // self.HK


@dataclass(frozen=True)
class Prefill:
    name: str
    B: int
    T: int
    H: int
    HK: int
    D: int
    theta: float

    @property
    def flops(self):
        return 4 * self.B * self.H * self.D * self.T * (self.T + 1) // 2

    @property
    def io_bytes(self):
        """Bytes the producer moves: F32 q/k/v in, F32 KV-cache rows out, BF16 q/k/v out."""
        per_tok = self.D * (4 * (self.H + 2 * self.HK) + 4 * 2 * self.HK + 2 * (self.H + 2 * self.HK))
        return self.B * self.T * per_tok


C2_B1 = Decode("llama3-8b decode B=1 ctx=4096", 1, 32, 8, 128, 4096, 500000.0)
C2_B8 = Decode("llama3-8b decode B=8 ctx=4096", 8, 32, 8, 128, 4096, 500000.0)
C2_B64 = Decode("llama3-8b decode B=64 ctx=4096", 64, 32, 8, 128, 4096, 500000.0)
C3 = Prefill("llama2-7b causal prefill B=4 T=2048", 4, 2048, 32, 32, 128, 10000.0)
C4 = Decode("llama3-70b decode B=16 ctx=32768 (kv-head shard)", 16, 64, 8, 128, 32768, 500000.0)
# The 70B-shaped decode at B=2: the per-GPU share of C4 on 8 GPUs (537 MB,
# one wave of CTAs) and the size the ncu captures of that kernel are taken at.
C4_SMALL = Decode("llama3-70b decode B=2 ctx=32768 (per-GPU share at 8 GPUs)", 2, 64, 8, 128, 32768, 500000.0)
C5 = Decode("long-context decode B=1 ctx=131072 (seq-chunk shard)", 1, 32, 8, 128, 131072, 500000.0)
C5_SMALL = Decode("long-context decode B=1 ctx=16384 (per-GPU share at 8 GPUs)", 1, 32, 8, 128, 16384, 500000.0)


def head_shard(w: Decode, world: int, rank: int):
    """KV heads [r*HK/N, (r+1)*HK/N) with their query heads; kv_head = h*HK/H
    (src/pickle_fast.c:1963) keeps every query head with its KV head."""
    if w.HK % world:
        raise ValueError(f"{w.HK} KV heads do not split {world} ways")
    hk = w.HK // world
    h = w.H // world
    return (rank * h, (rank + 1) * h), (rank * hk, (rank + 1) * hk)


def seq_shard(ctx: int, world: int, rank: int):
    """Cache positions [p0, p1) held by `rank` for a context of `ctx` rows;
    the new token (position ctx) is appended by the last rank."""
    per = (ctx + world - 1) // world
    p0 = min(rank * per, ctx)
    p1 = min(p0 + per, ctx)
    return p0, p1
