"""Python mirror of the C ABI in include/pickle_cuda.h (ctypes).

The attention block of pickle's forward pass
(lee-muriithi-kingori/lestramanika src/pickle_fast.c:1910-2109) runs in
libpickle_cuda.so; this module only loads it, declares the signatures and
turns pickle's negative status codes (src/pickle.h:52-60) into exceptions.
There is no fallback: if the library is missing, every call raises.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpickle_cuda.so")

PICKLE_OK = 0
ERROR_NAMES = {
    -1: "PICKLE_ERR_FORMAT", -2: "PICKLE_ERR_VERSION", -3: "PICKLE_ERR_MEMORY",
    -4: "PICKLE_ERR_TYPE", -5: "PICKLE_ERR_IO", -6: "PICKLE_ERR_ARG",
    -7: "PICKLE_ERR_RANGE", -8: "PICKLE_ERR_ARCH", -9: "PICKLE_ERR_DEVICE",
}
PREFILL_F32 = 0
PREFILL_BF16 = 1


class PickleError(RuntimeError):
    """A negative PICKLE_ERR_* status from the library."""

    def __init__(self, code, what="", detail=""):
        self.code = code
        name = ERROR_NAMES.get(code, str(code))
        super().__init__(f"{what}: {name}" + (f" ({detail})" if detail else ""))


class Params(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("max_seq", ctypes.c_int), ("half", ctypes.c_int),
        ("rope_inv_freq", ctypes.POINTER(ctypes.c_float)), ("rope_theta", ctypes.c_float),
        ("n_seqs", ctypes.c_int), ("rope_len", ctypes.c_int),
    ]


_lib = None
_vp, _fp, _i, _sz = ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_size_t
_i32p = ctypes.POINTER(ctypes.c_int32)

LAYER_TENSORS = 9   # PICKLE_CUDA_LAYER_TENSORS


class Tensor(ctypes.Structure):
    """pickle_cuda_tensor_t: one tensor's raw GGML bytes."""
    _fields_ = [("type", _i), ("data", _vp), ("nbytes", _sz)]


class ModelParams(ctypes.Structure):
    """pickle_cuda_model_params_t."""
    _fields_ = [
        ("n_layers", _i), ("hidden_dim", _i), ("intermediate_dim", _i),
        ("n_heads", _i), ("n_kv_heads", _i), ("head_dim", _i),
        ("vocab_size", _i), ("max_seq", _i),
        ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("rope_inv_freq", _fp),
        ("max_tokens", _i), ("prefill_precision", _i), ("weights_on_device", _i),
        ("token_embd", Tensor), ("output_norm", Tensor), ("output", Tensor),
        ("layers", ctypes.POINTER(Tensor)),
        ("n_seqs", _i),
    ]

SIGNATURES = {
    "pickle_cuda_abi_version": ([], _i),
    "pickle_cuda_init": ([ctypes.POINTER(Params), _i, ctypes.POINTER(_vp)], _i),
    "pickle_cuda_free": ([_vp], None),
    "pickle_cuda_attn_decode": ([_vp, _i, _sz, _fp, _fp, _fp, _fp], _i),
    "pickle_cuda_attn_prefill": ([_vp, _i, _sz, _sz, _fp, _fp, _fp, _fp, _i], _i),
    "pickle_cuda_decode_batch_dev": ([_vp, _i, _i, _sz, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_prefill_dev": ([_vp, _i, _i, _sz, _sz, _vp, _vp, _vp, _vp, _i, _vp], _i),
    "pickle_cuda_decode_partial_dev": ([_vp, _i, _i, _sz, _sz, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_lse_merge_dev": ([_i, _i, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_lse_merge_packed_dev": ([_i, _i, _i, _vp, _sz, _vp, _vp], _i),
    "pickle_cuda_kv_write": ([_vp, _i, _i, _sz, _sz, _fp, _fp], _i),
    "pickle_cuda_kv_layout": ([_vp, _i, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                               ctypes.POINTER(_sz), ctypes.POINTER(_sz)], _i),
    "pickle_cuda_sync": ([_vp, _vp], _i),
    "pickle_cuda_decode_plan": ([_vp, _i, _sz, ctypes.POINTER(_i), ctypes.POINTER(_i)], _i),
    "pickle_cuda_last_error": ([_vp], ctypes.c_char_p),
    "pickle_cuda_prefill_attn_bf16_dev": ([_i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_decode_noalloc": ([_i, _i, _i, _i, _i, _i, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp], _i),
    "pickle_cuda_decode_ragged_dev": ([_vp, _i, _i, _vp, _vp, _sz, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_prefill_slot_dev": ([_vp, _i, _i, _sz, _sz, _vp, _vp, _vp, _vp, _i, _vp], _i),
    "pickle_cuda_matvec_dev": ([_i, _vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "pickle_cuda_matvec_row_bytes": ([_i, _i], _sz),
    "pickle_cuda_matvec_take_error": ([_i, ctypes.POINTER(ctypes.c_int)], _i),
    "pickle_cuda_matmul_workspace": ([_i, _i, _i], _sz),
    "pickle_cuda_matmul_dev": ([_i, _vp, _i, _i, _i, _vp, _vp, _vp, _sz, _vp], _i),
    "pickle_cuda_model_load": ([ctypes.POINTER(ModelParams), _i, ctypes.POINTER(_vp)], _i),
    "pickle_cuda_model_free": ([_vp], None),
    "pickle_cuda_model_attn": ([_vp], _vp),
    "pickle_cuda_model_last_error": ([_vp], ctypes.c_char_p),
    "pickle_cuda_forward": ([_vp, _i32p, _sz, _fp, ctypes.POINTER(_sz)], _i),
    "pickle_cuda_forward_dev": ([_vp, _vp, _sz, _sz, _vp, _vp, _vp], _i),
    "pickle_cuda_forward_slot": ([_vp, _i, _i32p, _sz, _fp, ctypes.POINTER(_sz)], _i),
    "pickle_cuda_forward_batch_dev": ([_vp, _i, _vp, _vp, _vp, _sz, _vp, _vp, _vp], _i),
    "pickle_cuda_model_sync": ([_vp, _vp], _i),
    "pickle_cuda_argmax_dev": ([_vp, _i, _vp, _vp], _i),
    "pickle_cuda_sample_dev": ([_vp, _i, ctypes.c_float, ctypes.c_float, ctypes.c_uint32, _vp, _vp], _i),
    "pickle_cuda_generate_sampled": ([_vp, _i32p, _sz, _i, _i, ctypes.c_float, ctypes.c_float, ctypes.c_uint32,
                                      _i32p, ctypes.POINTER(_i), _fp, ctypes.POINTER(_sz)], _i),
    "pickle_cuda_generate": ([_vp, _i32p, _sz, _i, _i, _i32p, ctypes.POINTER(_i), _fp, ctypes.POINTER(_sz)], _i),
    "pickle_cuda_xchg_create": ([_i, _i, _sz, _i, ctypes.POINTER(_vp)], _i),
    "pickle_cuda_xchg_handle": ([_vp, _vp], _i),
    "pickle_cuda_xchg_open": ([_vp, _i, _vp], _i),
    "pickle_cuda_xchg_buffer": ([_vp, ctypes.POINTER(_vp)], _i),
    "pickle_cuda_xchg_put_dev": ([_vp, _vp, _sz, _sz, _sz, _sz, _sz, _vp], _i),
    "pickle_cuda_xchg_sync": ([_vp, _vp], _i),
    "pickle_cuda_xchg_last_error": ([_vp], ctypes.c_char_p),
    "pickle_cuda_xchg_free": ([_vp], None),
    "pickle_cuda_xchg_attach": ([_vp, _i, _vp], _i),
    "pickle_cuda_xchg_set_wait": ([_vp, ctypes.c_ulonglong], _i),
    "pickle_cuda_decode_gather_dev": ([_vp, _vp, _i, _i, _sz, _vp, _vp, _vp, _vp, _vp], _i),
    "pickle_cuda_decode_xchg_bytes": ([_i, _i, _i, _i, _i, ctypes.POINTER(_sz)], _i),
    "pickle_cuda_decode_seqshard_dev": ([_vp, _vp, _i, _i, _sz, _sz, _i, _vp, _vp, _vp, _vp, _vp], _i),
}

IPC_HANDLE_BYTES = 64


def lib():
    """Load libpickle_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run `python -m lestramanika_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_fp)


def _ptr(t):
    """Device address of a torch tensor (or an int address, or None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


class _DevArray:
    """Exposes a device address as __cuda_array_interface__ for torch.as_tensor."""

    def __init__(self, ptr, shape, owner):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": "<f4", "data": (ptr, False), "version": 3, "strides": None,
        }
        self._owner = owner


class PickleCuda:
    """One device KV cache + RoPE tables for a model's attention block.

    Mirrors pickle_cuda_t: the dimensions are those of
    pickle_fast_state_t (src/pickle_fast.h:55-123).
    """

    def __init__(self, n_layers, n_heads, n_kv_heads, head_dim, max_seq, *, half=None,
                 rope_inv_freq=None, rope_theta=10000.0, n_seqs=1, rope_len=0, device=0):
        self.n_layers, self.H, self.HK, self.D = n_layers, n_heads, n_kv_heads, head_dim
        self.max_seq, self.n_seqs, self.device = max_seq, n_seqs, device
        self.half = min(head_dim // 2, 64) if half is None else half
        self.rope_len = rope_len if rope_len else max_seq
        p = Params(n_layers, n_heads, n_kv_heads, head_dim, max_seq, self.half, None,
                   float(rope_theta), n_seqs, rope_len)
        if rope_inv_freq is not None:
            self._inv, p.rope_inv_freq = _f32(rope_inv_freq)
        h = _vp()
        rc = lib().pickle_cuda_init(ctypes.byref(p), device, ctypes.byref(h))
        if rc != PICKLE_OK:
            raise PickleError(rc, "pickle_cuda_init")
        self._h = h

    # -- helpers ---------------------------------------------------------
    def _check(self, rc, what):
        if rc != PICKLE_OK:
            msg = lib().pickle_cuda_last_error(self._h)
            raise PickleError(rc, what, msg.decode() if msg else "")

    def close(self):
        if getattr(self, "_h", None):
            lib().pickle_cuda_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- host-buffer entry points (what pickle_fast_forward calls) -------
    def attn_decode(self, layer, pos, q, k, v):
        q, qp = _f32(q)
        k, kp = _f32(k)
        v, vp = _f32(v)
        ao = np.empty(self.H * self.D, np.float32)
        self._check(lib().pickle_cuda_attn_decode(self._h, layer, pos, qp, kp, vp, ao.ctypes.data_as(_fp)),
                    "pickle_cuda_attn_decode")
        return ao

    def attn_prefill(self, layer, pos0, q, k, v, precision=PREFILL_F32):
        q, qp = _f32(q)
        k, kp = _f32(k)
        v, vp = _f32(v)
        T = q.size // (self.H * self.D)
        ao = np.empty((T, self.H * self.D), np.float32)
        self._check(lib().pickle_cuda_attn_prefill(self._h, layer, pos0, T, qp, kp, vp,
                                                   ao.ctypes.data_as(_fp), precision),
                    "pickle_cuda_attn_prefill")
        return ao

    def kv_write(self, layer, seq, pos0, k_rows, v_rows):
        k_rows, kp = _f32(k_rows)
        v_rows, vp = _f32(v_rows)
        n = k_rows.size // (self.HK * self.D)
        self._check(lib().pickle_cuda_kv_write(self._h, layer, seq, pos0, n, kp, vp), "pickle_cuda_kv_write")

    # -- device-buffer entry points (torch tensors / addresses) ----------
    def decode_batch_dev(self, layer, n_seqs, pos, q, k, v, ao, stream=None):
        self._check(lib().pickle_cuda_decode_batch_dev(self._h, layer, n_seqs, pos, _ptr(q), _ptr(k), _ptr(v),
                                                       _ptr(ao), _stream(stream)),
                    "pickle_cuda_decode_batch_dev")

    def decode_ragged_dev(self, layer, pos, q, k, v, ao, slots=None, max_pos=None, stream=None):
        """pickle_cuda_decode_ragged_dev: entry i (cache slot slots[i], or i) at its own
        position pos[i] (int32 device tensors); max_pos defaults to pos.max() (a host sync)."""
        if max_pos is None:
            max_pos = int(pos.max().item())
        self._check(lib().pickle_cuda_decode_ragged_dev(self._h, layer, int(pos.numel()), _ptr(pos), _ptr(slots),
                                                        max_pos, _ptr(q), _ptr(k), _ptr(v), _ptr(ao),
                                                        _stream(stream)),
                    "pickle_cuda_decode_ragged_dev")

    def prefill_slot_dev(self, layer, slot, pos0, T, q, k, v, ao, precision=PREFILL_F32, stream=None):
        self._check(lib().pickle_cuda_prefill_slot_dev(self._h, layer, slot, pos0, T, _ptr(q), _ptr(k), _ptr(v),
                                                       _ptr(ao), precision, _stream(stream)),
                    "pickle_cuda_prefill_slot_dev")

    def prefill_dev(self, layer, n_seqs, pos0, T, q, k, v, ao, precision=PREFILL_F32, stream=None):
        self._check(lib().pickle_cuda_prefill_dev(self._h, layer, n_seqs, pos0, T, _ptr(q), _ptr(k), _ptr(v),
                                                  _ptr(ao), precision, _stream(stream)),
                    "pickle_cuda_prefill_dev")

    def decode_partial_dev(self, layer, n_seqs, pos, n_local, append, q, k, v, m, l, acc, stream=None):
        self._check(lib().pickle_cuda_decode_partial_dev(self._h, layer, n_seqs, pos, n_local, int(bool(append)),
                                                         _ptr(q), _ptr(k), _ptr(v), _ptr(m), _ptr(l), _ptr(acc),
                                                         _stream(stream)),
                    "pickle_cuda_decode_partial_dev")

    def decode_gather_dev(self, xchg, layer, n_seqs, pos, q, k, v, out, stream=None):
        """pickle_cuda_decode_gather_dev: this rank's heads decoded and exchanged; out
        [n_seqs][world * H][D] receives every rank's head outputs."""
        self._check(lib().pickle_cuda_decode_gather_dev(self._h, xchg._x, layer, n_seqs, pos, _ptr(q), _ptr(k),
                                                        _ptr(v), _ptr(out), _stream(stream)),
                    "pickle_cuda_decode_gather_dev")

    def decode_seqshard_dev(self, xchg, layer, n_seqs, pos, n_local, append, q, k, v, out, stream=None):
        """pickle_cuda_decode_seqshard_dev: partial over this rank's n_local cache rows,
        triples exchanged with every rank and merged into out [n_seqs][H][D]."""
        self._check(lib().pickle_cuda_decode_seqshard_dev(self._h, xchg._x, layer, n_seqs, pos, n_local,
                                                          int(bool(append)), _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                          _stream(stream)),
                    "pickle_cuda_decode_seqshard_dev")

    def sync(self, stream=None):
        self._check(lib().pickle_cuda_sync(self._h, _stream(stream)), "pickle_cuda_sync")

    def decode_plan(self, n_seqs, pos):
        s, n = ctypes.c_int(), ctypes.c_int()
        self._check(lib().pickle_cuda_decode_plan(self._h, n_seqs, pos, ctypes.byref(s), ctypes.byref(n)),
                    "pickle_cuda_decode_plan")
        return s.value, n.value

    def kv_layout(self, layer):
        k, v, ss, hs = _vp(), _vp(), _sz(), _sz()
        self._check(lib().pickle_cuda_kv_layout(self._h, layer, ctypes.byref(k), ctypes.byref(v),
                                                ctypes.byref(ss), ctypes.byref(hs)), "pickle_cuda_kv_layout")
        return k.value, v.value, ss.value, hs.value

    def kv_tensors(self, layer):
        """Torch views [n_seqs][HK][max_seq][D] of layer `layer`'s K and V cache."""
        import torch
        k, v, _, _ = self.kv_layout(layer)
        shape = (self.n_seqs, self.HK, self.max_seq, self.D)
        dev = torch.device("cuda", self.device)
        return (torch.as_tensor(_DevArray(k, shape, self), device=dev),
                torch.as_tensor(_DevArray(v, shape, self), device=dev))


def lse_merge_dev(n_parts, n_rows, head_dim, m, l, acc, out, stream=None):
    rc = lib().pickle_cuda_lse_merge_dev(n_parts, n_rows, head_dim, _ptr(m), _ptr(l), _ptr(acc), _ptr(out),
                                         _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_lse_merge_dev")


def prefill_attn_bf16_dev(n_seqs, T, n_heads, n_kv_heads, head_dim, q, k, v, ao, err_flag=None, stream=None):
    """Causal attention on rotated BF16 head-major q/k/v (tensor cores), F32 output."""
    rc = lib().pickle_cuda_prefill_attn_bf16_dev(n_seqs, T, n_heads, n_kv_heads, head_dim, _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(ao), _ptr(err_flag), _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_prefill_attn_bf16_dev")


def decode_noalloc(n_seqs, n_heads, n_kv_heads, head_dim, half, max_seq, pos, rope_sin, rope_cos, q, k, v,
                   k_cache, v_cache, ao, err_flag=None, stream=None):
    """pickle_cuda_decode_noalloc on caller-owned device tensors (no allocation inside)."""
    rc = lib().pickle_cuda_decode_noalloc(n_seqs, n_heads, n_kv_heads, head_dim, half, max_seq, pos,
                                          _ptr(rope_sin), _ptr(rope_cos), _ptr(q), _ptr(k), _ptr(v),
                                          _ptr(k_cache), _ptr(v_cache), _ptr(ao), _ptr(err_flag), _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_decode_noalloc")


def lse_merge_packed_dev(n_parts, n_rows, head_dim, parts, part_stride, out, stream=None):
    rc = lib().pickle_cuda_lse_merge_packed_dev(n_parts, n_rows, head_dim, _ptr(parts), part_stride, _ptr(out),
                                                _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_lse_merge_packed_dev")


# GGML weight types the device matvec takes (src/pickle.h:85-97).
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 2, 8, 12, 14


def matvec_row_bytes(ggml_type, in_n):
    return lib().pickle_cuda_matvec_row_bytes(ggml_type, in_n)


def matvec_dev(ggml_type, W, out_n, in_n, x, y, n_vec=1, stream=None):
    """pickle_cuda_matvec_dev: y [n_vec][out_n] = W x for raw GGML weight bytes W (uint8 device tensor)."""
    rc = lib().pickle_cuda_matvec_dev(ggml_type, _ptr(W), out_n, in_n, n_vec, _ptr(x), _ptr(y), _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_matvec_dev")


def matmul_workspace(out_n, in_n, n_tok):
    """pickle_cuda_matmul_workspace: device bytes the batched matmul's tensor-core path needs."""
    return lib().pickle_cuda_matmul_workspace(out_n, in_n, n_tok)


def matmul_dev(ggml_type, W, out_n, in_n, x, y, n_tok, workspace=None, stream=None):
    """pickle_cuda_matmul_dev: y [n_tok][out_n] = x [n_tok][in_n] W^T for raw GGML weight bytes W.
    `workspace` (a uint8 device tensor of matmul_workspace(...) bytes) enables the tensor-core GEMM."""
    ws, nb = (None, 0) if workspace is None else (_ptr(workspace), workspace.numel() * workspace.element_size())
    rc = lib().pickle_cuda_matmul_dev(ggml_type, _ptr(W), out_n, in_n, n_tok, _ptr(x), _ptr(y), ws, nb,
                                      _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_matmul_dev")


def matvec_take_error(device=0):
    """pickle_cuda_matvec_take_error: the matvec's device error code (0 = none), cleared."""
    code = ctypes.c_int(0)
    rc = lib().pickle_cuda_matvec_take_error(device, ctypes.byref(code))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_matvec_take_error")
    return code.value


def argmax_dev(logits, out, stream=None):
    """pickle_fast_argmax on a device f32 vector into a device int32 (asynchronous)."""
    rc = lib().pickle_cuda_argmax_dev(_ptr(logits), logits.numel(), _ptr(out), _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_argmax_dev")


def sample_dev(logits, out, temp, top_p=0.0, seed=0, stream=None):
    """pickle_fast_sample_temp on a device f32 vector (overwritten with the
    exponentials when temp > 0) into a device int32 (asynchronous)."""
    rc = lib().pickle_cuda_sample_dev(_ptr(logits), logits.numel(), float(temp), float(top_p), int(seed) & 0xFFFFFFFF,
                                      _ptr(out), _stream(stream))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_sample_dev")


def abi_version():
    return lib().pickle_cuda_abi_version()


class PeerExchange:
    """pickle_cuda_xchg_t: one rank's side of the NVLink peer exchange of the
    sharded decodes (plain peer stores through CUDA IPC, no NCCL).

    Every rank creates one with the same buf_bytes, shares handle() with the
    others and open()s theirs; put() then writes this rank's rows into every
    rank's receive buffer (buffer()) and completes on the GPU when all ranks'
    rows of that call have arrived here.
    """

    def __init__(self, rank, world, buf_bytes, device=0):
        self.rank, self.world, self.buf_bytes, self.device = rank, world, buf_bytes, device
        h = _vp()
        rc = lib().pickle_cuda_xchg_create(rank, world, buf_bytes, device, ctypes.byref(h))
        if rc != PICKLE_OK:
            raise PickleError(rc, "pickle_cuda_xchg_create")
        self._x = h

    def _check(self, rc, what):
        if rc != PICKLE_OK:
            msg = lib().pickle_cuda_xchg_last_error(self._x)
            raise PickleError(rc, what, msg.decode() if msg else "")

    def handle(self):
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        self._check(lib().pickle_cuda_xchg_handle(self._x, buf), "pickle_cuda_xchg_handle")
        return buf.raw

    def open(self, peer, handle):
        buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
        self._check(lib().pickle_cuda_xchg_open(self._x, peer, buf), "pickle_cuda_xchg_open")

    def buffer(self, shape):
        """Torch float32 view of this rank's receive buffer."""
        import torch
        ptr = _vp()
        self._check(lib().pickle_cuda_xchg_buffer(self._x, ctypes.byref(ptr)), "pickle_cuda_xchg_buffer")
        return torch.as_tensor(_DevArray(ptr.value, shape, self), device=torch.device("cuda", self.device))

    def put(self, src, rows, row_bytes, src_stride, dst_offset, dst_stride, stream=None):
        self._check(lib().pickle_cuda_xchg_put_dev(self._x, _ptr(src), rows, row_bytes, src_stride, dst_offset,
                                                   dst_stride, _stream(stream)), "pickle_cuda_xchg_put_dev")

    def sync(self, stream=None):
        self._check(lib().pickle_cuda_xchg_sync(self._x, _stream(stream)), "pickle_cuda_xchg_sync")

    def attach(self, peer, other):
        """Use rank `peer`'s exchange `other`, made by this process, as that peer."""
        self._check(lib().pickle_cuda_xchg_attach(self._x, peer, other._x), "pickle_cuda_xchg_attach")

    def set_wait(self, wait_ns):
        """Bound of every flag wait of this exchange's kernels (ns)."""
        self._check(lib().pickle_cuda_xchg_set_wait(self._x, int(wait_ns)), "pickle_cuda_xchg_set_wait")

    def close(self):
        if self._x:
            lib().pickle_cuda_xchg_free(self._x)
            self._x = None


SHARD_HEADS, SHARD_SEQ = 0, 1


def decode_xchg_bytes(sharding, world, n_seqs, n_heads, head_dim):
    """pickle_cuda_decode_xchg_bytes: exchange buffer bytes of the fused sharded decodes
    (SHARD_HEADS: n_heads = this rank's query heads; SHARD_SEQ: all query heads)."""
    n = _sz()
    rc = lib().pickle_cuda_decode_xchg_bytes(sharding, world, n_seqs, n_heads, head_dim, ctypes.byref(n))
    if rc != PICKLE_OK:
        raise PickleError(rc, "pickle_cuda_decode_xchg_bytes")
    return n.value
