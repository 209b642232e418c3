"""Parity oracle for pickle's attention block - TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
use this package, and only as the checker (or the timed CPU baseline).
The product library never imports or links anything under oracle/.

* OracleAttn      - ctypes wrapper of liboracle_attn.so, the C restatement
                    of lee-muriithi-kingori/lestramanika src/pickle_fast.c:
                    1634-1640, 1772-1788 and 1910-2094 (ref_attn_cpu.c).
* RefBlock        - ctypes wrapper of _ref/libref_attn_block.so, the
                    reference's own attention block compiled from its
                    sources (present only where the reference was built).
* e2e_run         - runs one of the _ref/pickle_e2e_* token-id drivers.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
ORACLE_LIB = os.path.join(HERE, "liboracle_attn.so")
REF_BLOCK_LIB = os.path.join(REF_DIR, "libref_attn_block.so")

_fp = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p
_i, _sz = ctypes.c_int, ctypes.c_size_t


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_fp)


def half_of(D):
    """RoPE pairs per head, src/pickle_fast.c:1515-1516."""
    return min(D // 2, 64)


_olib = None


def oracle_lib():
    global _olib
    if _olib is None:
        if not os.path.exists(ORACLE_LIB):
            subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
        L = ctypes.CDLL(ORACLE_LIB)
        L.oracle_attn_create.argtypes = [_i, _i, _i, _i, _i, ctypes.c_float, ctypes.POINTER(_vp)]
        L.oracle_attn_create.restype = _i
        L.oracle_attn_destroy.argtypes = [_vp]
        L.oracle_attn_destroy.restype = None
        L.oracle_attn_decode.argtypes = [_vp, _i, _sz, _fp, _fp, _fp, _fp]
        L.oracle_attn_decode.restype = _i
        for n in ("oracle_attn_k_cache", "oracle_attn_v_cache", "oracle_attn_sin", "oracle_attn_cos",
                  "oracle_attn_inv_freq"):
            getattr(L, n).argtypes = [_vp]
            getattr(L, n).restype = _fp
        L.oracle_rope_tables.argtypes = [ctypes.c_float, _i, _i, _i, _fp, _fp, _fp]
        L.oracle_rope_tables.restype = _i
        L.oracle_attn_decode_batch.argtypes = [_i, _i, _i, _i, _i, _sz, _fp, _fp, _fp, _fp, _fp, _fp, _fp, _fp]
        L.oracle_attn_decode_batch.restype = _i
        L.oracle_attend_rows.argtypes = [_i, _i, _i, _sz, _fp, _fp, _fp, _fp]
        L.oracle_attend_rows.restype = _i
        L.oracle_rope_apply.argtypes = [_fp, _i, _i, _fp, _fp]
        L.oracle_rope_apply.restype = None
        _olib = L
    return _olib


def rope_tables(theta, D, n_pos):
    """(inv_freq [half], sin [n_pos][half], cos [n_pos][half]) as the reference builds them."""
    half = half_of(D)
    inv = np.zeros(max(half, 1), np.float32)
    s = np.zeros((n_pos, max(half, 1)), np.float32)
    c = np.zeros((n_pos, max(half, 1)), np.float32)
    rc = oracle_lib().oracle_rope_tables(theta, D, half, n_pos, inv.ctypes.data_as(_fp), s.ctypes.data_as(_fp),
                                         c.ctypes.data_as(_fp))
    assert rc == 0
    return inv[:half], s[:, :half], c[:, :half]


class OracleAttn:
    """Stateful oracle: one model's host KV cache, one token per call."""

    def __init__(self, n_layers, H, HK, D, max_seq, theta=10000.0):
        self.n_layers, self.H, self.HK, self.D, self.max_seq = n_layers, H, HK, D, max_seq
        h = _vp()
        rc = oracle_lib().oracle_attn_create(n_layers, H, HK, D, max_seq, theta, ctypes.byref(h))
        if rc != 0:
            raise ValueError(f"oracle_attn_create rc={rc}")
        self._h = h

    def decode(self, layer, pos, q, k, v):
        """Returns ao [H*D]; q/k are copied (the oracle rotates its copies)."""
        q, qp = _f32(np.array(q, np.float32, copy=True))
        k, kp = _f32(np.array(k, np.float32, copy=True))
        v, vp = _f32(v)
        ao = np.empty(self.H * self.D, np.float32)
        rc = oracle_lib().oracle_attn_decode(self._h, layer, pos, qp, kp, vp, ao.ctypes.data_as(_fp))
        if rc != 0:
            raise ValueError(f"oracle_attn_decode rc={rc}")
        return ao

    def cache(self, layer):
        """Views (K, V) [max_seq][HK][D] of this layer's pos-major cache."""
        L = oracle_lib()
        n = self.n_layers * self.max_seq * self.HK * self.D
        k = np.ctypeslib.as_array(L.oracle_attn_k_cache(self._h), shape=(n,))
        v = np.ctypeslib.as_array(L.oracle_attn_v_cache(self._h), shape=(n,))
        shp = (self.n_layers, self.max_seq, self.HK, self.D)
        return k.reshape(shp)[layer], v.reshape(shp)[layer]

    def close(self):
        if self._h:
            oracle_lib().oracle_attn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_batch(H, HK, D, pos, sin_row, cos_row, kc, vc, q, k, v):
    """Oracle batched decode over pos-major caches kc/vc [n_seqs][max_seq][HK][D].

    q [n_seqs][H][D], k/v [n_seqs][HK][D] (pre-RoPE). Writes the rotated k
    and v into kc/vc at `pos` and returns ao [n_seqs][H][D].
    """
    n_seqs, max_seq = kc.shape[0], kc.shape[1]
    assert kc.flags.c_contiguous and vc.flags.c_contiguous and kc.dtype == np.float32
    q = np.array(q, np.float32, copy=True, order="C")
    k = np.array(k, np.float32, copy=True, order="C")
    v = np.ascontiguousarray(v, np.float32)
    sr, sp = _f32(sin_row)
    cr, cp = _f32(cos_row)
    ao = np.empty((n_seqs, H, D), np.float32)
    rc = oracle_lib().oracle_attn_decode_batch(n_seqs, H, HK, D, max_seq, pos, sp, cp, kc.ctypes.data_as(_fp),
                                               vc.ctypes.data_as(_fp), q.ctypes.data_as(_fp),
                                               k.ctypes.data_as(_fp), v.ctypes.data_as(_fp),
                                               ao.ctypes.data_as(_fp))
    assert rc == 0, rc
    return ao


def attend_rows(q_rot, kc_rows, vc_rows, H, HK, D):
    """Attention of rotated q [H][D] over pos-major rows [n][HK][D] (no RoPE, no append)."""
    q_rot, qp = _f32(q_rot)
    kc_rows, kp = _f32(kc_rows)
    vc_rows, vp = _f32(vc_rows)
    n = kc_rows.size // (HK * D)
    ao = np.empty(H * D, np.float32)
    rc = oracle_lib().oracle_attend_rows(H, HK, D, n, kp, vp, qp, ao.ctypes.data_as(_fp))
    assert rc == 0
    return ao.reshape(H, D)


def rope_apply(x, D, sin_row, cos_row):
    """Rotate x [..., heads, D] in place-copy with one table row."""
    x = np.array(x, np.float32, copy=True, order="C")
    heads = x.size // D
    sr, sp = _f32(sin_row)
    cr, cp = _f32(cos_row)
    oracle_lib().oracle_rope_apply(x.ctypes.data_as(_fp), heads, D, sp, cp)
    return x


class RefBlock:
    """The reference's own attention block (oracle/_ref/libref_attn_block.so)."""

    _lib = None

    @classmethod
    def available(cls):
        return os.path.exists(REF_BLOCK_LIB)

    @classmethod
    def lib(cls):
        if cls._lib is None:
            L = ctypes.CDLL(REF_BLOCK_LIB)
            L.ref_block_new.argtypes = [_i, _i, _i, _i, _i, ctypes.c_float]
            L.ref_block_new.restype = _vp
            L.ref_block_decode.argtypes = [_vp, _i, _sz, _fp, _fp, _fp, _fp]
            L.ref_block_decode.restype = _i
            L.ref_block_free.argtypes = [_vp]
            L.ref_block_free.restype = None
            for n in ("ref_block_k_cache", "ref_block_v_cache"):
                getattr(L, n).argtypes = [_vp]
                getattr(L, n).restype = _fp
            cls._lib = L
        return cls._lib

    def __init__(self, n_layers, H, HK, D, max_seq, theta=10000.0):
        self.n_layers, self.H, self.HK, self.D, self.max_seq = n_layers, H, HK, D, max_seq
        self._h = self.lib().ref_block_new(n_layers, H, HK, D, max_seq, theta)
        if not self._h:
            raise MemoryError("ref_block_new")

    def decode(self, layer, pos, q, k, v):
        q, qp = _f32(np.array(q, np.float32, copy=True))
        k, kp = _f32(np.array(k, np.float32, copy=True))
        v, vp = _f32(np.array(v, np.float32, copy=True))
        ao = np.empty(self.H * self.D, np.float32)
        rc = self.lib().ref_block_decode(self._h, layer, pos, qp, kp, vp, ao.ctypes.data_as(_fp))
        if rc != 0:
            raise ValueError(f"ref_block_decode rc={rc}")
        return ao

    def cache(self, layer):
        """Views (K, V) [max_seq][HK][D] of the reference's pos-major cache."""
        n = self.n_layers * self.max_seq * self.HK * self.D
        k = np.ctypeslib.as_array(self.lib().ref_block_k_cache(self._h), shape=(n,))
        v = np.ctypeslib.as_array(self.lib().ref_block_v_cache(self._h), shape=(n,))
        shp = (self.n_layers, self.max_seq, self.HK, self.D)
        return k.reshape(shp)[layer], v.reshape(shp)[layer]

    def close(self):
        if self._h:
            self.lib().ref_block_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def e2e_binary(kind):
    """Path of the pickle_e2e driver linked with `kind` in {ref, oracle, cuda}."""
    return os.path.join(REF_DIR, f"pickle_e2e_{kind}")


def read_e2e(path):
    b = open(path, "rb").read()
    n_prompt, n = np.frombuffer(b[:8], np.int32)
    ids = np.frombuffer(b[8:8 + 4 * n], np.int32).copy()
    margins = np.frombuffer(b[8 + 4 * n:8 + 8 * n], np.float32).copy()
    vs = int(np.frombuffer(b[8 + 8 * n:12 + 8 * n], np.int32)[0])
    logits = np.frombuffer(b[12 + 8 * n:12 + 8 * n + 4 * vs], np.float32).copy()
    return {"n_prompt": int(n_prompt), "ids": ids, "margins": margins, "logits": logits}


def read_dump(path, H, HK, D):
    """Per hook call: (layer, pos, q, k, v, ao) from an e2e dump file."""
    nq, nk = H * D, HK * D
    rec = 2 + nq + 2 * nk + nq
    raw = np.fromfile(path, dtype=np.float32)
    assert raw.size % rec == 0
    raw = raw.reshape(-1, rec)
    hdr = raw[:, :2].copy().view(np.int32)
    q = raw[:, 2:2 + nq]
    k = raw[:, 2 + nq:2 + nq + nk]
    v = raw[:, 2 + nq + nk:2 + nq + 2 * nk]
    ao = raw[:, 2 + nq + 2 * nk:]
    return hdr[:, 0], hdr[:, 1], q, k, v, ao


def e2e_run(kind, model_path, out_path, n_gen, prompt, dump_path=None, env=None, timeout=600):
    exe = e2e_binary(kind)
    cmd = [exe, model_path, out_path, str(n_gen), dump_path or "-"] + [str(int(x)) for x in prompt]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{exe} rc={r.returncode}: {r.stderr.strip()[-500:]}")
    return read_e2e(out_path)
