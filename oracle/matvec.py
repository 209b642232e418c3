"""TEST INFRASTRUCTURE ONLY - CPU restatement of the reference's weight
matvec for the formats the device matvec takes, the checker of
lestramanika_b200/csrc/matvec.cu. Never imported by the product.

y[o] = sum_i w(o, i) * x[i], with w the float weight the reference computes
per element (lee-muriithi-kingori/lestramanika src/pickle_fast.c):
  F32   :122-146   w = W[o][i]
  F16   :1381-1419 w = half_to_float(W[o][i])
  Q4_0  :161-196   18-byte blocks of 32: d (f16), byte j -> element j
                   (low nibble) and 16 + j (high nibble); w = d * (q - 8)
  Q8_0  :303-326   34-byte blocks of 32: d (f16), 32 int8; w = d * q
  Q4_K  :563-738   144-byte blocks of 256: d, dmin (f16), 12 bytes of
                   6-bit scales/mins (:368-383), 128 bytes of nibbles in
                   4 chunks of 64; w = (d * sc) * q - dmin * m
  Q6_K  :1084-1257 210-byte blocks of 256: ql[128], qh[64], int8
                   scales[16], d (f16); w = (d * scale) * (q - 32)
The dequantized weights are formed in float32 with those expressions and
the dot products taken in float64. Pinned against the reference's own
kernels compiled from its sources (oracle/_ref/libref_matvec.so) by
tests/test_matvec_cpu.py.
"""
import ctypes
import os

import numpy as np

TYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14}
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 14: (256, 210)}   # (elements, bytes)


def row_bytes(t, in_n):
    qk, bb = BLOCK[t]
    return in_n // qk * bb


def _f16(b, off):
    return b[..., off:off + 2].copy().view(np.float16).astype(np.float32)[..., 0]


def dequant(t, W, out_n, in_n):
    """float32 [out_n][in_n] weights from the raw bytes W (uint8)."""
    W = np.asarray(W, np.uint8).reshape(out_n, row_bytes(t, in_n))
    if t == 0:
        return W.view(np.float32).reshape(out_n, in_n).copy()
    if t == 1:
        return W.view(np.float16).astype(np.float32).reshape(out_n, in_n)
    qk, bb = BLOCK[t]
    b = W.reshape(out_n, in_n // qk, bb)
    if t == 2:
        d = _f16(b, 0)[..., None]
        qs = b[..., 2:18].astype(np.int32)
        q = np.concatenate([qs & 15, qs >> 4], axis=-1) - 8
        return (d * q.astype(np.float32)).reshape(out_n, in_n).astype(np.float32)
    if t == 8:
        d = _f16(b, 0)[..., None]
        q = b[..., 2:34].view(np.int8).astype(np.float32)
        return (d * q).reshape(out_n, in_n).astype(np.float32)
    if t == 12:
        d = _f16(b, 0)
        dmin = _f16(b, 2)
        s = b[..., 4:16].astype(np.int32)
        sc = np.empty(b.shape[:-1] + (8,), np.int32)
        mn = np.empty_like(sc)
        for j in range(8):
            if j < 4:
                sc[..., j] = s[..., j] & 63
                mn[..., j] = s[..., j + 4] & 63
            else:
                sc[..., j] = (s[..., j + 4] & 15) | ((s[..., j - 4] >> 6) << 4)
                mn[..., j] = (s[..., j + 4] >> 4) | ((s[..., j] >> 6) << 4)
        qs = b[..., 16:144].astype(np.int32).reshape(out_n, in_n // 256, 4, 32)
        out = np.empty((out_n, in_n // 256, 4, 2, 32), np.float32)
        for c in range(4):
            for h in range(2):
                q = (qs[:, :, c] & 15) if h == 0 else (qs[:, :, c] >> 4)
                d1 = (d * sc[..., 2 * c + h].astype(np.float32)).astype(np.float32)[..., None]
                m1 = (dmin * mn[..., 2 * c + h].astype(np.float32)).astype(np.float32)[..., None]
                out[:, :, c, h] = (d1 * q.astype(np.float32) - m1).astype(np.float32)
        return out.reshape(out_n, in_n)
    if t == 14:
        ql = b[..., 0:128].astype(np.int32)
        qh = b[..., 128:192].astype(np.int32)
        scales = b[..., 192:208].view(np.int8).astype(np.float32)
        d = _f16(b, 208)
        out = np.empty((out_n, in_n // 256, 2, 4, 32), np.float32)
        for n in range(2):
            for t4 in range(4):
                lo = ql[..., 64 * n + 32 * (t4 & 1): 64 * n + 32 * (t4 & 1) + 32]
                lo = (lo & 15) if t4 < 2 else (lo >> 4)
                hi = (qh[..., 32 * n: 32 * n + 32] >> (2 * t4)) & 3
                q = (lo | (hi << 4)) - 32
                for half in range(2):
                    ds = (d * scales[..., 8 * n + half + 2 * t4]).astype(np.float32)[..., None]
                    out[:, :, n, t4, 16 * half:16 * half + 16] = (ds * q[..., 16 * half:16 * half + 16]
                                                                 .astype(np.float32)).astype(np.float32)
        return out.reshape(out_n, in_n)
    raise ValueError(t)


def matvec(t, W, out_n, in_n, x):
    """y [n_vec][out_n] (float64) for x [n_vec][in_n]."""
    w = dequant(t, W, out_n, in_n).astype(np.float64)
    return np.atleast_2d(np.asarray(x, np.float64)) @ w.T


def random_weights(t, out_n, in_n, rng):
    """Raw bytes of a random valid W: small float scales, random quants."""
    rb = row_bytes(t, in_n)
    if t == 0:
        return rng.standard_normal((out_n, in_n), dtype=np.float32).view(np.uint8).reshape(-1)
    if t == 1:
        return (rng.standard_normal((out_n, in_n)) * 0.5).astype(np.float16).view(np.uint8).reshape(-1)
    qk, bb = BLOCK[t]
    nb = out_n * (in_n // qk)
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    def put_f16(off, scale):
        b[:, off:off + 2] = (rng.uniform(0.25, 1.0, nb) * scale).astype(np.float16).view(np.uint8).reshape(nb, 2)
    if t in (2, 8):
        put_f16(0, 0.05)
    elif t == 12:
        put_f16(0, 0.02)
        put_f16(2, 0.01)
    elif t == 14:
        put_f16(208, 0.01)
    return b.reshape(-1)[: out_n * rb].copy()


_ref = None


def ref_lib():
    """The reference's own kernels (oracle/_ref/libref_matvec.so), or None."""
    global _ref
    if _ref is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_matvec.so")
        if not os.path.exists(path):
            return None
        _ref = ctypes.CDLL(path)
    return _ref


_REF_FN = {0: "pickle_fast_matmul_f32", 1: "pickle_fast_matmul_f16", 2: "pickle_fast_matmul_q4_0",
           8: "pickle_fast_matmul_q8_0", 12: "pickle_fast_matmul_q4_k", 14: "pickle_fast_matmul_q6_k"}


def ref_matvec(t, W, out_n, in_n, x):
    """y [out_n] float32 from the reference's kernel for one vector x."""
    lib = ref_lib()
    y = np.zeros(out_n, np.float32)
    W = np.ascontiguousarray(W, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    up = ctypes.POINTER(ctypes.c_ubyte)
    if t == 0:
        f = lib.pickle_fast_matmul_f32          # (y, W, x, out_n, in_n)
        f.argtypes = [fp, fp, fp, ctypes.c_int, ctypes.c_int]
        f(y.ctypes.data_as(fp), W.view(np.float32).ctypes.data_as(fp), x.ctypes.data_as(fp), out_n, in_n)
    else:
        f = getattr(lib, _REF_FN[t])            # (y, W, out_n, in_n, x)
        f.argtypes = [fp, up, ctypes.c_int, ctypes.c_int, fp]
        f(y.ctypes.data_as(fp), W.ctypes.data_as(up), out_n, in_n, x.ctypes.data_as(fp))
    return y
