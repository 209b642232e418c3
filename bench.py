#!/usr/bin/env python3
"""Benchmark of the B200 attention block for pickle (decode-attn KV GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline at every N: Llama-3-70B-shaped decode attention, B=16, ctx 32768
(4.3 GB of F32 KV cache, larger than L2, so no flush between steps).
  N = 1: the whole cache on one GPU (split-KV decode kernel + merge).
  N > 1: KV heads sharded N ways (1/N of the cache per GPU); the head
         outputs are exchanged over NVLink inside the decode's merge launch
         (plain peer stores, per-row flags). Strong scaling: total work
         fixed, time = max over ranks; rank 0 also decodes the whole
         problem on one GPU (parity reference and 1-GPU time).
Series at every N: long-context decode, ctx 131072 (seq-chunk shard at
N > 1: partial (m, l, acc) triples exchanged and merged by log-sum-exp in the
same fused launch). N = 1 extras: Llama-3-8B-shaped decode B=1/8/64, causal
prefill (TFLOP/s), the projection matvec/GEMM. Decode steps are replayed
from a captured CUDA graph.

One JSON line on rank 0. `--impl reference` times the reference's own
OpenMP attention block (oracle/_ref, compiled from its sources) on all host
cores, on the same workload: a step is one reference call per sequence,
cycling over distinct caches that total more than the host's L3. The
`cpu_baseline` of this arm's line runs the same code.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from lestramanika_b200.workloads import C2_B1, C2_B8, C2_B64, C3, C4, C4_SMALL, C5, C5_SMALL  # noqa: E402

MEASURED = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS = 6650.0, 1590.0
L2_FLUSH_BYTES = 512 << 20
L2_BYTES = 126 << 20


def peaks():
    try:
        m = json.load(open(MEASURED))
        return float(m["hbm_gbs"]), float(m["bf16_tflops"]), float(m.get("bf16_tflops_sustained", m["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def profile_traffic(name):
    """dram read+write bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.strip().split("\t")
        if len(parts) >= 2 and parts[0] == name:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = str(device_index)
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.idx], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx.append(float(p[2]))
            except ValueError:
                continue
            for n, val in zip(names, p[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

def _torch():
    import torch
    return torch


def make_decode_state(w, device, H=None, HK=None, B=None, ctx_rows=None, seed=0, n_layers=1):
    """Handle with seeded N(0,1) device caches (n_layers layers) for workload w (or a shard of it)."""
    torch = _torch()
    from lestramanika_b200 import PickleCuda
    H = H or w.H
    HK = HK or w.HK
    B = B or w.B
    rows = w.ctx if ctx_rows is None else ctx_rows
    cu = PickleCuda(n_layers, H, HK, w.D, rows + 1, rope_theta=w.theta, n_seqs=B, rope_len=w.ctx + 1,
                    device=device)
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)
    for layer in range(n_layers):
        kt, vt = cu.kv_tensors(layer)
        for b in range(B):
            kt[b, :, :rows].normal_(generator=g)
            vt[b, :, :rows].normal_(generator=g)
    dev = torch.device("cuda", device)
    q = torch.randn((B, H, w.D), generator=g, device=dev)
    k = torch.randn((B, HK, w.D), generator=g, device=dev)
    v = torch.randn((B, HK, w.D), generator=g, device=dev)
    ao = torch.empty((B, H, w.D), device=dev)
    torch.cuda.synchronize(device)
    return cu, q, k, v, ao


def time_decode(cu, w, q, k, v, ao, steps, warmup, flush=None, n_layers=1):
    """Device time of `steps` decode launches (ms list), CUDA events on the launching stream.
    Step i attends layer i % n_layers."""
    torch = _torch()
    st = torch.cuda.current_stream()
    for i in range(warmup):
        cu.decode_batch_dev(i % n_layers, q.shape[0], w.ctx, q, k, v, ao, st)
    cu.sync(st)
    if flush is None:
        # The K steps are captured once in a CUDA graph and replayed between
        # the events, as a serving loop replays its decode step.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for i in range(steps):
                cu.decode_batch_dev(i % n_layers, q.shape[0], w.ctx, q, k, v, ao, cs)
        graph.replay()
        cu.sync(st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        graph.replay()
        e1.record(st)
        cu.sync(st)
        del graph
        return [e0.elapsed_time(e1) / steps] * steps
    # L2 flushed before every step, outside its event pair. Nothing syncs
    # between steps: the decode launch is queued while the flush runs, so the
    # events time the kernel, not the host's launch latency.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in ev:
        flush.add_(1)
        e0.record(st)
        cu.decode_batch_dev(0, q.shape[0], w.ctx, q, k, v, ao, st)
        e1.record(st)
    cu.sync(st)
    return [e0.elapsed_time(e1) for e0, e1 in ev]


def time_decode_e2e(cu, w, q, k, v, ao, steps, warmup):
    """Same decode with every step's q/k/v copied in from pinned host memory and
    the output read back to pinned host memory inside the timed region."""
    torch = _torch()
    st = torch.cuda.current_stream()
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hao = torch.empty(ao.shape, dtype=ao.dtype).pin_memory()

    def step():
        q.copy_(hq, non_blocking=True)
        k.copy_(hk, non_blocking=True)
        v.copy_(hv, non_blocking=True)
        cu.decode_batch_dev(0, q.shape[0], w.ctx, q, k, v, ao, st)
        hao.copy_(ao, non_blocking=True)

    for _ in range(warmup):
        step()
    cu.sync(st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    cu.sync(st)
    ms = e0.elapsed_time(e1) / steps
    h2d = sum(x.numel() * 4 for x in (hq, hk, hv))
    return ms, h2d, hao.numel() * 4


def decode_line(w, device, steps, warmup, small):
    """small: the cache fits in L2, so steps rotate over layer caches totalling
    twice L2 (the headline for the line), and the same decode is also timed
    on one layer with L2 flushed by a 512 MB write before every step."""
    torch = _torch()
    n_layers = -(-2 * L2_BYTES // w.kv_bytes) if small else 1
    cu, q, k, v, ao = make_decode_state(w, device, n_layers=n_layers)
    times = time_decode(cu, w, q, k, v, ao, steps, warmup, None, n_layers)
    splits = cu.decode_plan(w.B, w.ctx)[0]
    ms = sum(times) / len(times)
    out = {"workload": w.name, "ms": ms, "GBps": w.kv_bytes / (ms * 1e-3) / 1e9, "splits": splits,
           "l2": (f"{n_layers} layer caches rotated ({n_layers * w.kv_bytes / 1e6:.0f} MB > L2)" if small
                  else "inputs larger than L2")}
    e2e = None
    if small:
        flush = torch.empty(L2_FLUSH_BYTES // 4, device=f"cuda:{device}")
        ft = time_decode(cu, w, q, k, v, ao, steps, warmup, flush)
        fms = sum(ft) / len(ft)
        out["l2_write_flushed"] = {"ms": fms, "GBps": w.kv_bytes / (fms * 1e-3) / 1e9}
        del flush
    else:
        e2e = time_decode_e2e(cu, w, q, k, v, ao, steps, warmup)
    cu.close()
    del q, k, v, ao
    torch.cuda.empty_cache()
    return out, e2e


def prefill_line(w, device, steps, warmup, precision):
    """Causal prefill: the whole pickle_cuda_prefill_dev call (RoPE/cast/KV-cache
    producer + attention) and, for BF16, the tensor-core attention kernel alone
    (pickle_cuda_prefill_attn_bf16_dev on BF16 head-major operands)."""
    torch = _torch()
    from lestramanika_b200 import PickleCuda, api
    dev = torch.device("cuda", device)
    cu = PickleCuda(1, w.H, w.HK, w.D, w.T, rope_theta=w.theta, n_seqs=w.B, device=device)
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    q = torch.randn((w.B, w.T, w.H, w.D), generator=g, device=dev)
    k = torch.randn((w.B, w.T, w.HK, w.D), generator=g, device=dev)
    v = torch.randn((w.B, w.T, w.HK, w.D), generator=g, device=dev)
    ao = torch.empty_like(q)
    st = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(warmup):
            fn()
        cu.sync(st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        cu.sync(st)
        return e0.elapsed_time(e1) / steps

    ms = timed(lambda: cu.prefill_dev(0, w.B, 0, w.T, q, k, v, ao, precision, st))
    out = {"workload": w.name, "precision": "bf16-tcgen05" if precision else "f32-cuda-core", "ms": ms,
           "TFLOPs": w.flops / (ms * 1e-3) / 1e12, "includes": "rope+cast+kv-cache write producer + attention",
           "flops_per_step": w.flops}
    if precision:
        qb = q.transpose(1, 2).contiguous().to(torch.bfloat16)
        kb = k.transpose(1, 2).contiguous().to(torch.bfloat16)
        vb = v.transpose(1, 2).contiguous().to(torch.bfloat16)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        ams = timed(lambda: api.prefill_attn_bf16_dev(w.B, w.T, w.H, w.HK, w.D, qb, kb, vb, ao, err, st))
        out["attn_ms"] = ams
        out["attn_TFLOPs"] = w.flops / (ams * 1e-3) / 1e12
        out["producer_ms"] = ms - ams
        out["producer_GBps"] = w.io_bytes / ((ms - ams) * 1e-3) / 1e9 if ms > ams else None
    cu.close()
    return out


MATVEC_SHAPE = (14336, 4096)        # Llama-3-8B FFN up/gate projection


def matvec_line(device, steps, warmup, types=("F16", "Q8_0", "Q6_K", "Q4_K", "Q4_0")):
    """Device weight matvec (pickle_cuda_matvec_dev) on the Llama-3-8B FFN
    up shape, one vector: weight GB/s. Steps rotate over enough weight copies
    to total twice L2 and are replayed from a CUDA graph."""
    torch = _torch()
    from lestramanika_b200 import api
    out_n, in_n = MATVEC_SHAPE
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    res = {}
    for name in types:
        t = getattr(api, "GGML_" + name)
        wbytes = api.matvec_row_bytes(t, in_n) * out_n
        copies = max(2, -(-2 * L2_BYTES // wbytes))
        if t == api.GGML_F16:
            w0 = torch.randn((out_n, in_n), device=dev, generator=gen).half().view(torch.uint8).reshape(-1)
        else:      # random quant bytes with small positive f16 block scales
            w0 = torch.randint(0, 256, (wbytes,), device=dev, dtype=torch.uint8, generator=gen)
            blk = {api.GGML_Q8_0: (34, (0,)), api.GGML_Q4_K: (144, (0, 2)), api.GGML_Q6_K: (210, (208,)),
                   api.GGML_Q4_0: (18, (0,))}[t]
            b = w0.view(-1, blk[0])
            for off in blk[1]:
                sc = (torch.rand((b.shape[0],), device=dev, generator=gen) * 0.02 + 0.005).half()
                b[:, off:off + 2] = sc.view(torch.uint8).view(-1, 2)
        Ws = [w0] + [w0.clone() for _ in range(copies - 1)]
        x = torch.randn((1, in_n), device=dev)
        y = torch.empty((1, out_n), device=dev)
        st = torch.cuda.current_stream()
        for i in range(warmup):
            api.matvec_dev(t, Ws[i % copies], out_n, in_n, x, y, 1, st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cs = torch.cuda.current_stream()
            for i in range(steps):
                api.matvec_dev(t, Ws[i % copies], out_n, in_n, x, y, 1, cs)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        res[name] = {"us": round(ms * 1e3, 2), "GBps": wbytes / (ms * 1e-3) / 1e9, "weight_bytes": wbytes,
                     "copies_rotated": copies}
        del g, Ws, w0
        torch.cuda.empty_cache()
    return {"shape": f"{out_n}x{in_n}", "n_vec": 1, "types": res}


MATMUL_SHAPE = (6144, 4096, 2048)   # Llama-3-8B fused QKV projection of a 2048-token prompt


def matmul_line(device, steps, warmup, types=("Q4_K", "Q8_0", "F16")):
    """Batched projection (pickle_cuda_matmul_dev, tensor-core GEMM) on the
    QKV shape: useful TFLOP/s (2 out_n in_n n_tok per call) and the rate of
    the tensor pipe, which also runs the hi/lo correction products (3 MMAs
    per k for quantized weights, 2 for F16). Timed per call, including the x
    split and row-scale pre-passes."""
    torch = _torch()
    from lestramanika_b200 import api
    out_n, in_n, n_tok = MATMUL_SHAPE
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(12)
    x = torch.randn((n_tok, in_n), device=dev, generator=gen)
    y = torch.empty((n_tok, out_n), device=dev)
    ws = torch.empty(api.matmul_workspace(out_n, in_n, n_tok), dtype=torch.uint8, device=dev)
    res = {}
    for name in types:
        t = getattr(api, "GGML_" + name)
        wbytes = api.matvec_row_bytes(t, in_n) * out_n
        if t == api.GGML_F16:
            W = torch.randn((out_n, in_n), device=dev, generator=gen).half().view(torch.uint8).reshape(-1)
        else:      # random quant bytes with small positive f16 block scales
            W = torch.randint(0, 256, (wbytes,), device=dev, dtype=torch.uint8, generator=gen)
            bb, offs = {api.GGML_Q8_0: (34, (0,)), api.GGML_Q4_K: (144, (0, 2))}[t]
            b = W.view(-1, bb)
            for off in offs:
                sc = (torch.rand((b.shape[0],), device=dev, generator=gen) * 0.02 + 0.005).half()
                b[:, off:off + 2] = sc.view(torch.uint8).view(-1, 2)
        st = torch.cuda.current_stream()
        for _ in range(warmup):
            api.matmul_dev(t, W, out_n, in_n, x, y, n_tok, workspace=ws, stream=st)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            api.matmul_dev(t, W, out_n, in_n, x, y, n_tok, workspace=ws, stream=st)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        flop = 2.0 * out_n * in_n * n_tok
        mult = 2 if t == api.GGML_F16 else 3
        res[name] = {"ms": round(ms, 4), "TFLOPs_useful": flop / (ms * 1e-3) / 1e12,
                     "TFLOPs_tensor_pipe": mult * flop / (ms * 1e-3) / 1e12, "mma_per_k16": mult}
        del W
    return {"shape": f"{out_n}x{in_n}, {n_tok} tokens", "types": res,
            "note": "per call: x hi/lo split + per-row weight scales (pre-passes) + GEMM"}


def matmul_batch_line(device, steps, warmup, shape=(28672, 4096, 32)):
    """The GEMM on a decode batch: Llama-3-8B gate|up (Q4_K) for 32 tokens,
    two weight copies used in turn (132 MB, above L2): us per call and the
    weight stream in GB/s."""
    torch = _torch()
    from lestramanika_b200 import api
    out_n, in_n, n_tok = shape
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(13)
    t = api.GGML_Q4_K
    wbytes = api.matvec_row_bytes(t, in_n) * out_n
    Ws = []
    for _ in range(2):
        W = torch.randint(0, 256, (wbytes,), device=dev, dtype=torch.uint8, generator=gen)
        b = W.view(-1, 144)
        for off in (0, 2):
            sc = (torch.rand((b.shape[0],), device=dev, generator=gen) * 2e-4 + 1e-4).half()
            b[:, off:off + 2] = sc.view(torch.uint8).view(-1, 2)
        Ws.append(W)
    x = torch.randn((n_tok, in_n), device=dev, generator=gen)
    y = torch.empty((n_tok, out_n), device=dev)
    ws = torch.empty(api.matmul_workspace(out_n, in_n, n_tok), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream()
    for i in range(warmup):
        api.matmul_dev(t, Ws[i % 2], out_n, in_n, x, y, n_tok, workspace=ws, stream=st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        api.matmul_dev(t, Ws[i % 2], out_n, in_n, x, y, n_tok, workspace=ws, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / steps * 1e3
    return {"shape": f"{out_n}x{in_n} Q4_K, {n_tok} tokens", "us_per_call": us, "weight_GBps": wbytes / us / 1e3}


def matmul_cpu_baseline(types=("Q4_K", "Q8_0", "F16"), seconds=2.0):
    """The reference's own per-token projection (oracle/_ref matvec kernels,
    OpenMP on the host cores) on the QKV shape: ms per token, a bounded
    sample of tokens timed and the prompt's time extrapolated."""
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import matvec as mv
    if mv.ref_lib() is None:
        return {"unavailable": "oracle/_ref/libref_matvec.so not built"}
    out_n, in_n, n_tok = MATMUL_SHAPE
    res = {}
    for name in types:
        t = mv.TYPES[name]
        W = mv.random_weights(t, out_n, in_n, np.random.default_rng(t))
        x = np.random.default_rng(1).standard_normal(in_n, dtype=np.float32)
        mv.ref_matvec(t, W, out_n, in_n, x)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / len(types):
            mv.ref_matvec(t, W, out_n, in_n, x)
            n += 1
        ms_tok = (time.perf_counter() - t0) / n * 1e3
        res[name] = {"ms_per_token": ms_tok, "ms_per_prompt": ms_tok * n_tok, "tokens_timed": n,
                     "TFLOPs": 2.0 * out_n * in_n / (ms_tok * 1e-3) / 1e12}
    return {"kind": "reference", "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
            "sample": f"one token per call, {n_tok}-token prompt extrapolated", "types": res}


# Llama-3-8B attention half of one layer for a 2048-token prompt (hidden
# 4096, 32 query heads, 8 KV heads, head dim 128), Q4_K weights.
PL_SHAPE = dict(hidden=4096, H=32, HK=8, D=128, T=2048, wtype="Q4_K", theta=500000.0)


def prefill_layer_line(device, steps, warmup):
    """LayerPrefill (q/k/v GEMMs -> RoPE, cache append, BF16 tensor-core
    causal attention -> output GEMM) for one prompt: ms per layer and prompt
    tokens per second per layer."""
    torch = _torch()
    from lestramanika_b200 import PREFILL_BF16, PickleCuda, api
    from lestramanika_b200.prefill_layer import LayerPrefill
    c = PL_SHAPE
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(21)
    t = getattr(api, "GGML_" + c["wtype"])
    qd, kd = c["H"] * c["D"], c["HK"] * c["D"]

    def weights(out_n, in_n):
        W = torch.randint(0, 256, (api.matvec_row_bytes(t, in_n) * out_n,), device=dev, dtype=torch.uint8,
                          generator=gen)
        b = W.view(-1, 144)
        for off in (0, 2):
            sc = (torch.rand((b.shape[0],), device=dev, generator=gen) * 0.002 + 0.0005).half()
            b[:, off:off + 2] = sc.view(torch.uint8).view(-1, 2)
        return (t, W)

    cu = PickleCuda(1, c["H"], c["HK"], c["D"], c["T"] + 8, rope_theta=c["theta"], device=device)
    lp = LayerPrefill(cu, weights(qd, c["hidden"]), weights(kd, c["hidden"]), weights(kd, c["hidden"]),
                      weights(c["hidden"], qd), hidden=c["hidden"], max_tokens=c["T"])
    x = torch.randn((c["T"], c["hidden"]), device=dev, generator=gen) * 0.05
    out = torch.empty((c["T"], c["hidden"]), device=dev)
    st = torch.cuda.current_stream()
    for _ in range(warmup):
        lp.run(0, 0, x, out, PREFILL_BF16, st)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        lp.run(0, 0, x, out, PREFILL_BF16, st)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    cu.close()
    flop_proj = 2.0 * c["T"] * c["hidden"] * (2 * qd + 2 * kd)
    flop_attn = 4.0 * c["D"] * c["H"] * c["T"] * (c["T"] + 1) / 2
    return {"workload": "llama3-8b attention half of one layer, %d-token prompt, %s weights, BF16 attention"
                        % (c["T"], c["wtype"]),
            "ms_per_layer": round(ms, 4), "prompt_tokens_per_s": c["T"] / (ms * 1e-3),
            "TFLOPs_useful": (flop_proj + flop_attn) / (ms * 1e-3) / 1e12}


def prefill_layer_cpu(seconds=6.0):
    """The reference's own token-by-token cost of the same work on the host
    cores: its matvec kernels for the four projections of one token, and its
    attention block (oracle/_ref) at sampled positions of the prompt;
    extrapolated to the prompt."""
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    import numpy as np
    sys.path.insert(0, ROOT)
    import oracle
    from oracle import matvec as mv
    if mv.ref_lib() is None or not oracle.RefBlock.available():
        return {"unavailable": "oracle/_ref libraries not built"}
    c = PL_SHAPE
    t = mv.TYPES[c["wtype"]]
    qd, kd = c["H"] * c["D"], c["HK"] * c["D"]
    rng = np.random.default_rng(3)
    proj_ms = 0.0
    for out_n, in_n in ((qd, c["hidden"]), (kd, c["hidden"]), (kd, c["hidden"]), (c["hidden"], qd)):
        W = mv.random_weights(t, out_n, in_n, rng)
        xv = rng.standard_normal(in_n, dtype=np.float32)
        mv.ref_matvec(t, W, out_n, in_n, xv)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 8:
            mv.ref_matvec(t, W, out_n, in_n, xv)
            n += 1
        proj_ms += (time.perf_counter() - t0) / n * 1e3
    blk = oracle.RefBlock(1, c["H"], c["HK"], c["D"], c["T"] + 1, c["theta"])
    lib = oracle.RefBlock.lib()
    n_el = (c["T"] + 1) * c["HK"] * c["D"]
    np.ctypeslib.as_array(lib.ref_block_k_cache(blk._h), shape=(n_el,))[:] = rng.standard_normal(n_el, dtype=np.float32)
    np.ctypeslib.as_array(lib.ref_block_v_cache(blk._h), shape=(n_el,))[:] = rng.standard_normal(n_el, dtype=np.float32)
    q = rng.standard_normal(qd, dtype=np.float32)
    k = rng.standard_normal(kd, dtype=np.float32)
    v = rng.standard_normal(kd, dtype=np.float32)
    positions = np.linspace(0, c["T"] - 1, 16).astype(int)
    blk.decode(0, int(positions[-1]), q, k, v)
    t0 = time.perf_counter()
    for p in positions:
        blk.decode(0, int(p), q, k, v)
    attn_ms = (time.perf_counter() - t0) / len(positions) * 1e3
    blk.close()
    per_tok = proj_ms + attn_ms
    return {"kind": "reference", "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
            "sample": "one token's four projections, attention at 16 positions spread over the prompt",
            "ms_per_token": per_tok, "ms_per_layer": per_tok * c["T"], "projections_ms_per_token": proj_ms,
            "attention_ms_per_token": attn_ms}


FW_SHAPE = dict(n_layers=32, hidden=4096, ffn=14336, H=32, HK=8, D=128, vocab=128256, max_seq=4096, prompt=2048,
                n_gen=64, theta=500000.0)
# Q4_K_M-like mix (the per-tensor choice of llama.cpp's Q4_K_M files); token_embd F16, norms F32
FW_MIX = dict(attn_q="Q4_K", attn_k="Q4_K", attn_v="Q6_K", attn_output="Q4_K", ffn_gate="Q4_K", ffn_up="Q4_K",
              ffn_down="Q6_K", output="Q6_K")


def _fw_model(device, c):
    """Synthetic Llama-3-8B-shaped weights generated on the device (raw GGML
    blocks, random quants, block scales giving weights of a few hundredths)
    and a PickleModel over them."""
    torch = _torch()
    from lestramanika_b200 import api
    from lestramanika_b200.model import PickleModel
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(33)
    HD, ID, VS, qd, kd = c["hidden"], c["ffn"], c["vocab"], c["H"] * c["D"], c["HK"] * c["D"]
    scale_at = {"Q4_K": ((0, 1e-4, 3e-4), (2, 1e-4, 3e-4)), "Q6_K": ((208, 1e-5, 3e-5),)}

    def quant(name, *shape):
        """One allocation for same-type matrices that follow each other
        (q|k, gate|up), as the model packs them; -> a view per matrix."""
        t = getattr(api, "GGML_" + name)
        sizes = [api.matvec_row_bytes(t, i) * o for o, i in shape]
        W = torch.randint(0, 256, (sum(sizes),), device=dev, dtype=torch.uint8, generator=gen)
        b = W.view(-1, 144 if name == "Q4_K" else 210)
        for off, lo, hi in scale_at[name]:
            sc = (torch.rand((b.shape[0],), device=dev, generator=gen) * (hi - lo) + lo).half()
            b[:, off:off + 2] = sc.view(torch.uint8).view(-1, 2)
        out, o0 = [], 0
        for n in sizes:
            out.append((t, W[o0:o0 + n]))
            o0 += n
        return out

    def norm():
        return (0, (1.0 + 0.1 * torch.randn(HD, device=dev, generator=gen)).contiguous())

    shapes = {"attn_q": (qd, HD), "attn_k": (kd, HD), "attn_v": (kd, HD), "attn_output": (HD, qd),
              "ffn_gate": (ID, HD), "ffn_up": (ID, HD), "ffn_down": (HD, ID)}
    t = {"token_embd.weight": (1, (torch.randn((VS, HD), device=dev, generator=gen) * 0.02).half()),
         "output_norm.weight": norm(), "output.weight": quant(FW_MIX["output"], (VS, HD))[0]}
    groups = [("attn_q", "attn_k"), ("attn_v",), ("attn_output",), ("ffn_gate", "ffn_up"), ("ffn_down",)]
    for L in range(c["n_layers"]):
        t[f"blk.{L}.attn_norm.weight"] = norm()
        t[f"blk.{L}.ffn_norm.weight"] = norm()
        for grp in groups:
            assert len({FW_MIX[n] for n in grp}) == 1
            for n, w in zip(grp, quant(FW_MIX[grp[0]], *[shapes[n] for n in grp])):
                t[f"blk.{L}.{n}.weight"] = w
    arch = dict(n_layers=c["n_layers"], hidden_dim=HD, intermediate_dim=ID, n_heads=c["H"], n_kv_heads=c["HK"],
                head_dim=c["D"], vocab_size=VS, max_seq=c["max_seq"], rms_eps=1e-5, rope_theta=c["theta"])
    weight_bytes = sum(v[1].numel() * v[1].element_size() for k, v in t.items() if k != "token_embd.weight")
    return t, arch, weight_bytes


def forward_line(device, steps, warmup):
    """The whole forward pass on the device (pickle_cuda_model_*), Llama-3-8B
    shape, Q4_K_M-like weights: a 2048-token prompt through all 32 layers
    (GEMMs + BF16 causal attention), then greedy decode steps at context
    2048+ (matvecs + split-KV decode + argmax, the id fed back on the
    device); and the same through the host API pickle_cuda_generate (prompt
    from host memory, ids and logits back)."""
    torch = _torch()
    from lestramanika_b200 import PREFILL_BF16
    from lestramanika_b200.model import PickleModel
    c = FW_SHAPE
    dev = torch.device("cuda", device)
    tensors, arch, wbytes = _fw_model(device, c)
    m = PickleModel(tensors, arch, device=device, max_tokens=c["prompt"], precision=PREFILL_BF16)
    g = torch.Generator()
    g.manual_seed(5)
    prompt = torch.randint(3, c["vocab"], (c["prompt"],), generator=g, dtype=torch.int32)
    tok = prompt.to(dev)
    logits = torch.empty(c["vocab"], device=dev)
    nxt = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.Stream(device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # prefill
    for _ in range(warmup):
        m.forward_dev(tok, 0, logits, nxt, stream=st)
    m.sync(stream=st)
    n_pf = max(2, min(steps, 5))
    e0.record(st)
    for _ in range(n_pf):
        m.forward_dev(tok, 0, logits, nxt, stream=st)
    e1.record(st)
    m.sync(stream=st)
    pf_ms = e0.elapsed_time(e1) / n_pf
    # decode: n_gen greedy steps after the prompt, ids fed back on the device
    n_dec = c["n_gen"]
    for i in range(max(warmup, 3)):
        m.forward_dev(nxt, c["prompt"] + i, logits, nxt, stream=st)
    m.sync(stream=st)
    m.forward_dev(tok, 0, logits, nxt, stream=st)
    e0.record(st)
    for i in range(n_dec):
        m.forward_dev(nxt, c["prompt"] + i, logits, nxt, stream=st)
    e1.record(st)
    m.sync(stream=st)
    dec_ms = e0.elapsed_time(e1) / n_dec
    # end to end through the host API
    m.generate(prompt.numpy(), 4)
    t0 = time.perf_counter()
    ids, _, pos = m.generate(prompt.numpy(), n_dec)
    e2e_s = time.perf_counter() - t0
    m.close()
    kv_bytes = 2 * c["n_layers"] * c["HK"] * c["D"] * 4 * (c["prompt"] + n_dec / 2)   # f32 cache read per step
    dec_bytes = wbytes + c["hidden"] * 2 + kv_bytes
    return {"workload": "llama3-8b forward, Q4_K_M-like weights (synthetic, on device), %d-token prompt with "
                        "BF16 causal attention, then %d greedy decode steps" % (c["prompt"], n_dec),
            "prefill_ms": round(pf_ms, 3), "prefill_tokens_per_s": c["prompt"] / (pf_ms * 1e-3),
            "decode_ms_per_token": round(dec_ms, 4), "decode_tokens_per_s": 1e3 / dec_ms,
            "decode_bytes_per_token": dec_bytes, "decode_GBps": dec_bytes / (dec_ms * 1e-3) / 1e9,
            "weight_bytes": wbytes,
            "e2e_generate": {"s": e2e_s, "n_prompt": c["prompt"], "n_gen": int(len(ids)), "kv_pos": int(pos),
                             "h2d_bytes": c["prompt"] * 4, "d2h_bytes": int(len(ids)) * 4 + c["vocab"] * 4,
                             "tokens_per_s": (c["prompt"] + len(ids)) / e2e_s}}


def forward_decode_line(device, steps, warmup):
    """Decode steps of the device forward alone (Llama-3-8B shape,
    Q4_K_M-like weights) at context 2048 of the device cache, which holds
    zeros (the step reads the same bytes whatever they hold): the command the
    per-kernel launch list of a decode step is taken with."""
    torch = _torch()
    from lestramanika_b200.model import PickleModel
    c = FW_SHAPE
    dev = torch.device("cuda", device)
    tensors, arch, wbytes = _fw_model(device, c)
    m = PickleModel(tensors, arch, device=device, max_tokens=16)
    logits = torch.empty(c["vocab"], device=dev)
    nxt = torch.full((1,), 7, dtype=torch.int32, device=dev)
    st = torch.cuda.Stream(device=dev)
    P = c["prompt"]
    for i in range(warmup):
        m.forward_dev(nxt, P + i, logits, nxt, stream=st)
    m.sync(stream=st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        m.forward_dev(nxt, P + i, logits, nxt, stream=st)
    e1.record(st)
    m.sync(stream=st)
    ms = e0.elapsed_time(e1) / steps
    m.close()
    return {"workload": "llama3-8b decode steps at context %d, Q4_K_M-like weights" % P, "ms_per_token": ms,
            "tokens_per_s": 1e3 / ms, "weight_bytes": wbytes}


def forward_batch_line(device, steps, warmup, batches=(8, 32)):
    """Continuous-batching decode through the whole model (Llama-3-8B shape,
    Q4_K_M-like weights): one step decodes B sequences, each in its own
    cache slot at context 2048+ (the slots hold zeros: a step reads the same
    bytes whatever they hold), all B rows sharing each pass over the weights
    (pickle_cuda_forward_batch_dev with argmax ids). Tokens/s = B / step."""
    torch = _torch()
    from lestramanika_b200.model import PickleModel
    c = FW_SHAPE
    dev = torch.device("cuda", device)
    tensors, arch, wbytes = _fw_model(device, c)
    out = {"workload": "llama3-8b batched decode at context %d, Q4_K_M-like weights, B sequences per step"
                       % c["prompt"], "batches": {}}
    for B in batches:
        m = PickleModel(tensors, arch, device=device, max_tokens=16, n_seqs=B)
        logits = torch.empty((B, c["vocab"]), device=dev)
        nxt = torch.full((B,), 7, dtype=torch.int32, device=dev)
        slots = torch.arange(B, dtype=torch.int32, device=dev)
        st = torch.cuda.Stream(device=dev)
        P = c["prompt"]
        pos = [torch.full((B,), P + i, dtype=torch.int32, device=dev) for i in range(warmup + steps)]
        torch.cuda.synchronize()
        for i in range(warmup):
            m.forward_batch_dev(nxt, pos[i], slots, P + i, logits, nxt, stream=st)
        m.sync(stream=st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(warmup, warmup + steps):
            m.forward_batch_dev(nxt, pos[i], slots, P + i, logits, nxt, stream=st)
        e1.record(st)
        m.sync(stream=st)
        ms = e0.elapsed_time(e1) / steps
        m.close()
        kv = 2 * c["n_layers"] * c["HK"] * c["D"] * 4 * (P + warmup + steps / 2) * B
        out["batches"][str(B)] = {"ms_per_step": round(ms, 4), "tokens_per_s": B / (ms * 1e-3),
                                  "GBps": (wbytes + kv) / (ms * 1e-3) / 1e9}
    return out


def forward_cpu(seconds=8.0):
    """The reference's own per-token cost of the same forward on the host
    cores: its matvec kernels (oracle/_ref) for every projection shape and
    type of one layer and for the lm_head, and its attention block at
    context 2048; one token = 32 layers of that + the lm_head. The reference
    runs the prompt through the same per-token loop."""
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    import numpy as np
    sys.path.insert(0, ROOT)
    import oracle
    from oracle import matvec as mv
    if mv.ref_lib() is None or not oracle.RefBlock.available():
        return {"unavailable": "oracle/_ref libraries not built"}
    c = FW_SHAPE
    HD, ID, qd, kd = c["hidden"], c["ffn"], c["H"] * c["D"], c["HK"] * c["D"]
    shapes = {"attn_q": (qd, HD), "attn_k": (kd, HD), "attn_v": (kd, HD), "attn_output": (HD, qd),
              "ffn_gate": (ID, HD), "ffn_up": (ID, HD), "ffn_down": (HD, ID), "output": (c["vocab"], HD)}
    rng = np.random.default_rng(4)
    ms = {}
    for n, (out_n, in_n) in shapes.items():
        t = mv.TYPES[FW_MIX[n]]
        W = mv.random_weights(t, out_n, in_n, rng)
        xv = rng.standard_normal(in_n, dtype=np.float32)
        mv.ref_matvec(t, W, out_n, in_n, xv)
        k, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 10 or k < 2:
            mv.ref_matvec(t, W, out_n, in_n, xv)
            k += 1
        ms[n] = (time.perf_counter() - t0) / k * 1e3
        del W
    P = c["prompt"]
    blk = oracle.RefBlock(1, c["H"], c["HK"], c["D"], P + 1, c["theta"])
    lib = oracle.RefBlock.lib()
    n_el = (P + 1) * c["HK"] * c["D"]
    np.ctypeslib.as_array(lib.ref_block_k_cache(blk._h), shape=(n_el,))[:] = rng.standard_normal(n_el, dtype=np.float32)
    np.ctypeslib.as_array(lib.ref_block_v_cache(blk._h), shape=(n_el,))[:] = rng.standard_normal(n_el, dtype=np.float32)
    q, k_, v = (rng.standard_normal(d, dtype=np.float32) for d in (qd, kd, kd))
    blk.decode(0, P, q, k_, v)
    t0 = time.perf_counter()
    for _ in range(8):
        blk.decode(0, P, q, k_, v)
    attn_ms = (time.perf_counter() - t0) / 8 * 1e3
    blk.close()
    layer_ms = sum(v for n, v in ms.items() if n != "output") + attn_ms
    tok_ms = c["n_layers"] * layer_ms + ms["output"]
    return {"kind": "reference", "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
            "sample": "one token: each projection shape/type of a layer once, attention at context 2048, "
                      "lm_head; x 32 layers",
            "decode_ms_per_token": tok_ms, "decode_tokens_per_s": 1e3 / tok_ms,
            "prefill_ms_upper": P * tok_ms, "projection_ms": ms, "attention_ms_at_2048": attn_ms}


def matvec_cpu_baseline(types=("F16", "Q8_0", "Q6_K", "Q4_K", "Q4_0"), seconds=2.0):
    """The reference's own matvec kernels (oracle/_ref, OpenMP on all host
    cores) on the same shape: weight GB/s."""
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    import numpy as np
    sys.path.insert(0, ROOT)
    from oracle import matvec as mv
    if mv.ref_lib() is None:
        return {"unavailable": "oracle/_ref/libref_matvec.so not built"}
    out_n, in_n = MATVEC_SHAPE
    res = {}
    for name in types:
        t = mv.TYPES[name]
        W = mv.random_weights(t, out_n, in_n, np.random.default_rng(t))
        x = np.random.default_rng(1).standard_normal(in_n, dtype=np.float32)
        mv.ref_matvec(t, W, out_n, in_n, x)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / len(types):
            mv.ref_matvec(t, W, out_n, in_n, x)
            n += 1
        dt = time.perf_counter() - t0
        res[name] = {"GBps": W.nbytes * n / dt / 1e9, "calls": n}
    return {"kind": "reference", "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)),
            "types": res}


REF_CACHE_BYTES = 1 << 30     # distinct host caches cycled through by the CPU reference: above the host's L3


def host_cpu():
    """The host's CPU model (first /proc/cpuinfo entry), for the baseline record."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def config_of(w):
    """The workload description both arms print (identical dicts)."""
    return {"workload": w.name, "B": w.B, "H": w.H, "HK": w.HK, "D": w.D, "ctx": w.ctx,
            "l2": "inputs larger than L2 (no flush)"}


def ref_decode(w, steps, warmup):
    """The reference's own OpenMP attention block (oracle/_ref/libref_attn_block.so,
    compiled from its sources; the C restatement when that is not built) on
    all host cores, on workload w: the reference has no batch dimension, so
    a step is w.B calls, one per sequence at position ctx, each parallel over
    heads (src/pickle_fast.c:1960). The block is made with R layers and call i
    uses layer i % R, so the calls cycle over R distinct caches of
    >= 1 GiB in all - more than the host's L3. The `--impl reference` arm
    and the `cpu_baseline` of this arm's line both run this function."""
    ncores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(ncores)
    os.environ.setdefault("OMP_PROC_BIND", "close")
    import numpy as np
    import oracle
    per_layer = 2 * (w.ctx + 1) * w.HK * w.D * 4
    R = max(1, -(-REF_CACHE_BYTES // per_layer))
    if oracle.RefBlock.available():
        blk, kind = oracle.RefBlock(R, w.H, w.HK, w.D, w.ctx + 1, w.theta), "reference"
    else:
        blk, kind = oracle.OracleAttn(R, w.H, w.HK, w.D, w.ctx + 1, w.theta), "port"
    rng = np.random.Generator(np.random.Philox(5))
    k0, v0 = blk.cache(0)
    k0[:w.ctx] = rng.standard_normal(k0[:w.ctx].shape, dtype=np.float32)
    v0[:w.ctx] = rng.standard_normal(v0[:w.ctx].shape, dtype=np.float32)
    for L in range(1, R):          # distinct memory, same distribution: rows rotated
        kL, vL = blk.cache(L)
        kL[:w.ctx] = np.roll(k0[:w.ctx], 97 * L, axis=0)
        vL[:w.ctx] = np.roll(v0[:w.ctx], 97 * L, axis=0)
    q = rng.standard_normal(w.H * w.D, dtype=np.float32)
    k = rng.standard_normal(w.HK * w.D, dtype=np.float32)
    v = rng.standard_normal(w.HK * w.D, dtype=np.float32)
    i = 0
    for _ in range(warmup):
        for _ in range(w.B):
            blk.decode(i % R, w.ctx, q, k, v)
            i += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        for _ in range(w.B):
            blk.decode(i % R, w.ctx, q, k, v)
            i += 1
    dt = time.perf_counter() - t0
    blk.close()
    return {"value": w.kv_bytes * steps / dt / 1e9, "unit": "GB/s", "cores": ncores, "kind": kind,
            "ms_per_step": dt / steps * 1e3, "cpu": host_cpu(),
            "sample": f"{steps} whole steps of {w.name}: {w.B} calls each, one per sequence, cycling over "
                      f"{R} distinct {per_layer / 1e6:.0f} MB caches ({R * per_layer / 1e9:.2f} GB)"}


def prefill_cpu(w, n_pos=16):
    """The reference's prefill of workload w on all host cores: it runs a
    prompt token by token through its attention block (src/pickle_fast.c:1881),
    so one layer's prefill of B prompts of T tokens is B * T block calls at
    positions 0..T-1. Timed at n_pos positions spread over the prompt and
    extrapolated (the call's cost grows linearly with the position)."""
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    os.environ.setdefault("OMP_PROC_BIND", "close")
    import numpy as np
    import oracle
    if oracle.RefBlock.available():
        blk, kind = oracle.RefBlock(1, w.H, w.HK, w.D, w.T + 1, w.theta), "reference"
    else:
        blk, kind = oracle.OracleAttn(1, w.H, w.HK, w.D, w.T + 1, w.theta), "port"
    rng = np.random.Generator(np.random.Philox(9))
    kc, vc = blk.cache(0)
    kc[:w.T] = rng.standard_normal(kc[:w.T].shape, dtype=np.float32)
    vc[:w.T] = rng.standard_normal(vc[:w.T].shape, dtype=np.float32)
    q = rng.standard_normal(w.H * w.D, dtype=np.float32)
    k = rng.standard_normal(w.HK * w.D, dtype=np.float32)
    v = rng.standard_normal(w.HK * w.D, dtype=np.float32)
    pos = np.linspace(0, w.T - 1, n_pos).astype(int)
    blk.decode(0, int(pos[-1]), q, k, v)
    t0 = time.perf_counter()
    for p in pos:
        blk.decode(0, int(p), q, k, v)
    per_call = (time.perf_counter() - t0) / n_pos
    blk.close()
    ms = per_call * w.B * w.T * 1e3
    return {"value": w.flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "kind": kind,
            "cores": int(os.environ["OMP_NUM_THREADS"]), "cpu": host_cpu(),
            "sample": f"{n_pos} block calls at positions spread over the {w.T}-token prompt, "
                      f"extrapolated to {w.B} x {w.T} calls"}


def _decode_extra(w, device, steps, warmup, small, hbm):
    line, _ = decode_line(w, device, steps, warmup, small)
    line["frac_of_measured_hbm"] = line["GBps"] / hbm
    return line


def run_ours_single(args):
    torch = _torch()
    device = 0
    torch.cuda.set_device(device)
    hbm, bf16, bf16_sus, src = peaks()
    w = C4
    with ClockSampler(device) as clk:
        head, e2e = decode_line(w, device, args.steps, args.warmup, small=False)
    extras = {}
    # The long-context series' 1-GPU point and the small-batch decodes.
    c5 = _decode_extra(C5, device, max(args.steps, 5), args.warmup, False, hbm)
    extras["c5_series"] = {"workload": C5.name, "n_gpus": 1, "ms": c5["ms"], "GBps": c5["GBps"],
                           "roofline_frac_per_gpu": c5["frac_of_measured_hbm"], "splits": c5["splits"]}
    for wx, small in ((C2_B64, False), (C2_B8, False), (C2_B1, True), (C4_SMALL, False)):
        extras[wx.name] = _decode_extra(wx, device, max(args.steps, 5), args.warmup, small, hbm)
    try:
        from lestramanika_b200 import PREFILL_BF16
        pf = prefill_line(C3, device, max(5, min(args.steps, 10)), max(args.warmup, 3), PREFILL_BF16)
        pf["roofline"] = {"bound": "tensor", "achieved": pf["TFLOPs"], "peak": bf16, "unit": "TFLOP/s",
                          "frac": pf["TFLOPs"] / bf16, "peak_source": f"{src} (bf16_tflops, cuBLAS burst)"}
        pf["attn_roofline"] = {"bound": "tensor", "achieved": pf["attn_TFLOPs"], "peak": bf16, "unit": "TFLOP/s",
                               "frac": pf["attn_TFLOPs"] / bf16}
        if not args.no_cpu_baseline:
            pf["cpu_baseline"] = prefill_cpu(C3)
        extras["prefill"] = pf
    except Exception as exc:  # reported, not hidden
        extras["prefill"] = {"error": str(exc)[:200]}
    try:
        mvl = matvec_line(device, max(args.steps, 20), max(args.warmup, 3))
        for r in mvl["types"].values():
            r["frac_of_measured_hbm"] = r["GBps"] / hbm
        extras["matvec"] = mvl
    except Exception as exc:  # reported, not hidden
        extras["matvec"] = {"error": str(exc)[:200]}
    try:
        mml = matmul_line(device, max(min(args.steps, 10), 3), max(args.warmup, 3))
        for r in mml["types"].values():
            r["frac_of_measured_bf16_tensor"] = r["TFLOPs_tensor_pipe"] / bf16
        extras["matmul"] = mml
    except Exception as exc:  # reported, not hidden
        extras["matmul"] = {"error": str(exc)[:200]}
    try:
        extras["prefill_layer"] = prefill_layer_line(device, max(min(args.steps, 10), 3), max(args.warmup, 3))
    except Exception as exc:  # reported, not hidden
        extras["prefill_layer"] = {"error": str(exc)[:200]}
    gbps = head["GBps"]
    e2e_ms, h2d, d2h = e2e
    out = {
        "metric": "decode-attn KV GB/s", "value": gbps, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) cache and q/k/v, seeded",
        "config": config_of(w),
        "parallelism": "single GPU", "splits": head["splits"],
        "frac_of_8TBps": gbps / 8000.0,
        "roofline": {"bound": "hbm", "achieved": gbps, "peak": hbm, "unit": "GB/s", "frac": gbps / hbm,
                     "peak_source": f"{src} (hbm_gbs, copy burst)",
                     "traffic": profile_traffic("decode_splitkv C4 B=16"),
                     "algorithmic_bytes_per_launch": w.kv_bytes},
        "e2e": {"value": w.kv_bytes / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": args.steps * (2 if head["splits"] > 1 else 1),   # split kernel (+ merge kernel)
        "clocks": clk.summary(),
        "extras": extras,
    }
    if not args.no_cpu_baseline:
        # The reference arm's code on a shorter run (whole steps of the same workload).
        out["cpu_baseline"] = ref_decode(w, min(args.steps, 8), 1)
    print(json.dumps(out), flush=True)


def run_ours_multi(args, rank, world, local_rank):
    torch = _torch()
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local_rank))
    from lestramanika_b200 import dist as pdist
    hbm, _, _, src = peaks()
    w = C4
    clk = ClockSampler(local_rank) if rank == 0 else None
    if clk:
        clk.__enter__()
    try:
        res = pdist.bench_head_sharded(w, rank, world, local_rank, args.steps, args.warmup)
    finally:
        if clk:
            clk.__exit__(None, None, None)
    res_seq = pdist.bench_seq_sharded(C5, rank, world, local_rank, args.steps, args.warmup)
    if rank == 0:
        gbps = w.kv_bytes / (res["ms"] * 1e-3) / 1e9
        one = res["one_gpu"]
        one5 = res_seq["one_gpu"]
        out = {
            "metric": "decode-attn KV GB/s", "value": gbps, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) cache and q/k/v, seeded",
            "config": config_of(w),
            "parallelism": f"kv-head shard x{world}, head outputs exchanged over NVLink inside the merge launch",
            "splits": res["splits"],
            "frac_of_8TBps_per_gpu": gbps / world / 8000.0,
            "roofline": {"bound": "hbm", "achieved": res["kernel_GBps_per_gpu"], "peak": hbm, "unit": "GB/s",
                         "frac": res["kernel_GBps_per_gpu"] / hbm, "peak_source": f"{src} (hbm_gbs)",
                         "traffic": None, "note": "per-GPU split-KV decode kernel alone (its 1/N of the cache)"},
            "e2e": res["e2e"],
            "gpu_launches": args.steps * res["launches_per_step"],   # per rank: split + fused merge/exchange
            "clocks": clk.summary() if clk else {"sm_mhz": None, "reasons": ["unsampled"]},
            "parity": {"max_rel_err_vs_one_gpu": one["max_rel_err_vs_one_gpu"], "bar": 1e-4,
                       "reference": "the whole problem decoded on GPU 0 from the same seeded shards"},
            "extras": {
                "one_gpu_ms": one["one_gpu_ms"],
                "builder_efficiency": one["one_gpu_ms"] / (world * res["ms"]),
                "nccl_all_gather": {"ms": res["nccl_all_gather_ms"],
                                    "GBps": w.kv_bytes / (res["nccl_all_gather_ms"] * 1e-3) / 1e9},
                "c5_series": {"workload": C5.name, "n_gpus": world, "ms": res_seq["ms"],
                              "GBps": C5.kv_bytes / (res_seq["ms"] * 1e-3) / 1e9,
                              "roofline_frac_per_gpu": res_seq["kernel_GBps_per_gpu"] / hbm,
                              "kernel_ms": res_seq["kernel_ms"],
                              "nccl_all_gather_ms": res_seq["nccl_all_gather_ms"],
                              "one_gpu_ms": one5["one_gpu_ms"],
                              "builder_efficiency": one5["one_gpu_ms"] / (world * res_seq["ms"]),
                              "max_rel_err_vs_one_gpu": one5["max_rel_err_vs_one_gpu"]}},
        }
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


ONLY = {"c2b1": (C2_B1, True), "c2b8": (C2_B8, False), "c2b64": (C2_B64, False), "c4": (C4, False),
        "c4s": (C4_SMALL, False), "c5": (C5, False), "c5s": (C5_SMALL, False), "c3": (C3, None), "mv": (None, None), "mm": (None, None),
        "pl": (None, None), "fw": (None, None), "fwd": (None, None), "fwb": (None, None),
        "fwb32": (None, None), "mmb": (None, None)}


def run_only(args):
    """One workload, one GPU: the command the ncu summaries under profiles/ were taken with."""
    torch = _torch()
    torch.cuda.set_device(0)
    w, flush = ONLY[args.only]
    if args.only == "mv":
        line = matvec_line(0, args.steps, args.warmup)
        line["cpu_reference"] = matvec_cpu_baseline()
    elif args.only == "pl":
        line = prefill_layer_line(0, args.steps, args.warmup)
        line["cpu_reference"] = prefill_layer_cpu()
        if "ms_per_layer" in line["cpu_reference"]:
            line["speedup_vs_reference"] = line["cpu_reference"]["ms_per_layer"] / line["ms_per_layer"]
    elif args.only == "fw":
        line = forward_line(0, args.steps, args.warmup)
        line["cpu_reference"] = forward_cpu()
        ref = line["cpu_reference"]
        if "decode_ms_per_token" in ref:
            line["decode_speedup_vs_reference"] = ref["decode_ms_per_token"] / line["decode_ms_per_token"]
    elif args.only == "fwd":
        line = forward_decode_line(0, args.steps, args.warmup)
    elif args.only == "fwb":
        line = forward_batch_line(0, args.steps, args.warmup)
    elif args.only == "mmb":
        line = matmul_batch_line(0, args.steps, args.warmup)
    elif args.only == "fwb32":
        line = forward_batch_line(0, args.steps, args.warmup, batches=(32,))
    elif args.only == "mm":
        line = matmul_line(0, args.steps, args.warmup)
        line["cpu_reference"] = matmul_cpu_baseline()
        for k, r in line["types"].items():
            ref = line["cpu_reference"].get("types", {}).get(k)
            if ref:
                r["speedup_vs_reference"] = ref["ms_per_prompt"] / r["ms"]
    elif flush is None:
        from lestramanika_b200 import PREFILL_BF16
        line = prefill_line(w, 0, args.steps, args.warmup, PREFILL_BF16)
    else:
        line, _ = decode_line(w, 0, args.steps, args.warmup, flush)
    print(json.dumps({"only": args.only, **line}), flush=True)


def run_reference(args, rank):
    """The reference's own CPU attention block on the host cores (rank 0 only;
    other ranks exit without work): the same workload, metric and config as
    this arm's line at every N."""
    if rank != 0:
        return
    w = C4
    r = ref_decode(w, args.steps, args.warmup)
    out = {"impl": "reference", "metric": "decode-attn KV GB/s", "value": r["value"], "unit": "GB/s",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic N(0,1) cache and q/k/v, seeded", "config": config_of(w),
           "cpu_baseline": {"value": r["value"], "unit": "GB/s", "cores": r["cores"], "kind": r["kind"],
                            "sample": r["sample"], "cpu": r["cpu"]},
           "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=sorted(ONLY), help="run one workload on one GPU (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.only:
        run_only(args)
        return
    if world > 1:
        run_ours_multi(args, rank, world, local_rank)
    else:
        run_ours_single(args)


if __name__ == "__main__":
    main()
