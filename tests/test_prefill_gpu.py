"""Batched causal prefill on the GPU against T sequential oracle steps
(the reference prefills token by token, src/pickle_fast.c:1881)."""
import numpy as np
import pytest
import torch

import oracle
from gpu_util import BF16_ABS_TOL, assert_rel, normal
from lestramanika_b200 import PREFILL_BF16, PREFILL_F32, PickleCuda

pytestmark = pytest.mark.gpu


def _oracle_prefill(H, HK, D, S, theta, q, k, v, pos0=0, pre=None):
    o = oracle.OracleAttn(1, H, HK, D, S, theta)
    if pre is not None:
        for p, (qq, kk, vv) in enumerate(pre):
            o.decode(0, p, qq, kk, vv)
    out = np.stack([o.decode(0, pos0 + t, q[t], k[t], v[t]) for t in range(q.shape[0])])
    kc, vc = o.cache(0)
    kc, vc = kc.copy(), vc.copy()
    o.close()
    return out, kc, vc


@pytest.mark.parametrize("H,HK,D,T", [(6, 6, 48, 37), (8, 2, 128, 70), (32, 8, 128, 129), (16, 2, 64, 33)])
def test_prefill_f32_host_api(H, HK, D, T):
    theta = 10000.0
    q = normal(5, (T, H * D), 1)
    k = normal(5, (T, HK * D), 2)
    v = normal(5, (T, HK * D), 3)
    cu = PickleCuda(1, H, HK, D, T + 8, rope_theta=theta)
    got = cu.attn_prefill(0, 0, q, k, v, PREFILL_F32)
    ref, kc, vc = _oracle_prefill(H, HK, D, T + 8, theta, q, k, v)
    assert_rel(got, ref, what=f"prefill H={H} HK={HK} D={D} T={T}")
    # decode continues from the cache the prefill wrote
    qn, kn, vn = normal(6, H * D, 1), normal(6, HK * D, 2), normal(6, HK * D, 3)
    got_d = cu.attn_decode(0, T, qn, kn, vn)
    o = oracle.OracleAttn(1, H, HK, D, T + 8, theta)
    for t in range(T):
        o.decode(0, t, q[t], k[t], v[t])
    assert_rel(got_d, o.decode(0, T, qn, kn, vn), what="decode after prefill")
    o.close()
    cu.close()


def test_prefill_f32_after_history():
    """Chunked prefill: T tokens at pos0 > 0 attend the earlier cache rows too."""
    H, HK, D, theta = 8, 2, 128, 10000.0
    pre = [(normal(8, H * D, p, 1), normal(8, HK * D, p, 2), normal(8, HK * D, p, 3)) for p in range(40)]
    T = 25
    q, k, v = normal(9, (T, H * D), 1), normal(9, (T, HK * D), 2), normal(9, (T, HK * D), 3)
    cu = PickleCuda(1, H, HK, D, 80, rope_theta=theta)
    for p, (qq, kk, vv) in enumerate(pre):
        cu.attn_decode(0, p, qq, kk, vv)
    got = cu.attn_prefill(0, 40, q, k, v, PREFILL_F32)
    ref, _, _ = _oracle_prefill(H, HK, D, 80, theta, q, k, v, pos0=40, pre=pre)
    assert_rel(got, ref, what="prefill after 40 rows")
    cu.close()


def test_prefill_batched_dev_writes_cache():
    B, T, H, HK, D, theta = 3, 50, 8, 8, 128, 10000.0
    q, k, v = normal(10, (B, T, H, D), 1), normal(10, (B, T, HK, D), 2), normal(10, (B, T, HK, D), 3)
    cu = PickleCuda(1, H, HK, D, T, rope_theta=theta, n_seqs=B)
    dev = torch.device("cuda", 0)
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    ao = torch.empty((B, T, H, D), dtype=torch.float32, device=dev)
    cu.prefill_dev(0, B, 0, T, qd, kd, vd, ao, PREFILL_F32)
    cu.sync()
    kt, vt = cu.kv_tensors(0)
    for b in range(B):
        ref, kc, vc = _oracle_prefill(H, HK, D, T, theta, q[b].reshape(T, -1), k[b].reshape(T, -1), v[b].reshape(T, -1))
        assert_rel(ao[b].cpu().numpy().reshape(T, -1), ref, what=f"seq {b}")
        np.testing.assert_allclose(kt[b].permute(1, 0, 2).cpu().numpy(), kc, atol=1e-5, rtol=0)
        np.testing.assert_array_equal(vt[b].permute(1, 0, 2).cpu().numpy(), vc)
    cu.close()


@pytest.mark.parametrize("H,HK,T", [(32, 32, 256), (8, 2, 300)])
def test_prefill_bf16(H, HK, T):
    """BF16 tensor-core prefill within 2e-2 max-abs of the F32 oracle."""
    D, theta = 128, 10000.0
    q = normal(11, (T, H * D), 1)
    k = normal(11, (T, HK * D), 2)
    v = normal(11, (T, HK * D), 3)
    cu = PickleCuda(1, H, HK, D, T, rope_theta=theta)
    got = cu.attn_prefill(0, 0, q, k, v, PREFILL_BF16)
    cu.close()
    ref, _, _ = _oracle_prefill(H, HK, D, T, theta, q, k, v)
    err = float(np.max(np.abs(got - ref)))
    assert err <= BF16_ABS_TOL, err


def test_prefill_bf16_full_length_subset_of_heads():
    """Llama-2-7B-shaped prefill length (T=2048, 32 MHA heads) on one sequence:
    every head runs on the GPU; heads 0, 13 and 31 are checked against the
    oracle (heads are independent when H == HK)."""
    H, HK, D, T, theta = 32, 32, 128, 2048, 10000.0
    q = normal(12, (T, H, D), 1)
    k = normal(12, (T, HK, D), 2)
    v = normal(12, (T, HK, D), 3)
    cu = PickleCuda(1, H, HK, D, T, rope_theta=theta)
    got = cu.attn_prefill(0, 0, q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1), PREFILL_BF16).reshape(T, H, D)
    cu.close()
    for h in (0, 13, 31):
        ref, _, _ = _oracle_prefill(1, 1, D, T, theta, q[:, h], k[:, h], v[:, h])
        err = float(np.max(np.abs(got[:, h] - ref)))
        assert err <= BF16_ABS_TOL, (h, err)


@pytest.mark.parametrize("B,T,H,HK", [(2, 384, 4, 2), (1, 200, 8, 8), (3, 300, 4, 4)])
def test_prefill_attn_bf16_entry_matches_torch_fp32(B, T, H, HK):
    """pickle_cuda_prefill_attn_bf16_dev against a plain PyTorch fp32 causal
    attention of the same BF16 operands."""
    from lestramanika_b200 import api
    D = 128
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    q = torch.randn((B, H, T, D), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((B, HK, T, D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((B, HK, T, D), generator=g, device=dev).to(torch.bfloat16)
    ao = torch.empty((B, T, H, D), device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    api.prefill_attn_bf16_dev(B, T, H, HK, D, q, k, v, ao, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    kk = k.float().repeat_interleave(H // HK, dim=1)
    vv = v.float().repeat_interleave(H // HK, dim=1)
    s = (q.float() @ kk.transpose(-1, -2)) / np.sqrt(np.float32(D))
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=dev), diagonal=1)
    ref = torch.softmax(s.masked_fill(mask, float("-inf")), dim=-1) @ vv        # [B][H][T][D]
    err_abs = float((ao.permute(0, 2, 1, 3) - ref).abs().max())
    assert err_abs <= 1e-2, err_abs


def test_prefill_bf16_batched_long_prompt_matches_f32_path():
    """A batched full-length GQA prompt (B=2, T=2048, 8 query / 4 KV heads):
    the KV cache the tensor-core path writes equals the F32 path's bit for
    bit, and every output row of every head is within the BF16 bar of the
    F32 path (itself checked against the oracle above)."""
    B, T, H, HK, D, theta = 2, 2048, 8, 4, 128, 10000.0
    dev = torch.device("cuda", 0)
    q, k, v = normal(13, (B, T, H, D), 1), normal(13, (B, T, HK, D), 2), normal(13, (B, T, HK, D), 3)
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    outs, caches = [], []
    for precision in (PREFILL_F32, PREFILL_BF16):
        cu = PickleCuda(1, H, HK, D, T, rope_theta=theta, n_seqs=B)
        ao = torch.full((B, T, H, D), float("nan"), device=dev)
        cu.prefill_dev(0, B, 0, T, qd, kd, vd, ao, precision)
        cu.sync()
        kt, vt = cu.kv_tensors(0)
        outs.append(ao.cpu().numpy())
        caches.append((kt.cpu().numpy(), vt.cpu().numpy()))
        cu.close()
    np.testing.assert_array_equal(caches[1][0], caches[0][0])
    np.testing.assert_array_equal(caches[1][1], caches[0][1])
    assert np.isfinite(outs[1]).all()
    err = float(np.max(np.abs(outs[1] - outs[0])))
    assert err <= BF16_ABS_TOL, err


def test_prefill_bf16_exact_c3_config_against_oracle():
    """The benchmark's prefill configuration as a whole: B=4 sequences x
    T=2048 tokens x 32 MHA heads (Llama-2-7B-shaped), one pickle_cuda_prefill_dev
    call on the tensor cores. Two heads of every sequence (a different pair
    per sequence) are checked against the oracle's token-by-token prefill
    (src/pickle_fast.c:1881 over :1910-2094) within the BF16 bar, and the
    KV-cache rows the call wrote for those heads equal the oracle's rotated k
    (1e-5) and v (exactly)."""
    B, T, H, HK, D, theta = 4, 2048, 32, 32, 128, 10000.0
    dev = torch.device("cuda", 0)
    q, k, v = normal(14, (B, T, H, D), 1), normal(14, (B, T, HK, D), 2), normal(14, (B, T, HK, D), 3)
    qd, kd, vd = (torch.from_numpy(x).to(dev) for x in (q, k, v))
    cu = PickleCuda(1, H, HK, D, T, rope_theta=theta, n_seqs=B)
    ao = torch.full((B, T, H, D), float("nan"), device=dev)
    cu.prefill_dev(0, B, 0, T, qd, kd, vd, ao, PREFILL_BF16)
    cu.sync()
    kt, vt = cu.kv_tensors(0)
    got = ao.cpu().numpy()
    assert np.isfinite(got).all()
    for b, heads in enumerate(((0, 31), (7, 20), (13, 26), (3, 17))):
        for h in heads:
            ref, kc, vc = _oracle_prefill(1, 1, D, T, theta, q[b, :, h], k[b, :, h], v[b, :, h])
            err = float(np.max(np.abs(got[b, :, h] - ref)))
            assert err <= BF16_ABS_TOL, (b, h, err)
            np.testing.assert_allclose(kt[b, h].cpu().numpy(), kc[:, 0], atol=1e-5, rtol=0)
            np.testing.assert_array_equal(vt[b, h].cpu().numpy(), vc[:, 0])
    cu.close()
