"""Minimal GGUF v3 reader: metadata and each tensor's raw bytes.

Reads the container the reference loads with pickle_load_from_file_mmap
(lee-muriithi-kingori/lestramanika src/pickle.c): the header (magic "GGUF",
version 3, tensor count, metadata count), the typed metadata key/values,
the tensor infos (name, dims with ne[0] the contiguous dimension, GGML type,
offset) and the tensor data, which starts at the next multiple of
general.alignment (32 by default) after the infos. Tensor bytes are
returned as read-only numpy views of a memory map, untouched: the device
path takes the raw GGML blocks as they are on disk.

Also arch_detect(), which reads the llama.* keys with the defaults of
pickle_arch_detect (src/pickle.c:988-1036).
"""
import struct

import numpy as np

# GGML type -> (bytes per block, elements per block)
BLOCK = {
    0: (4, 1), 1: (2, 1), 2: (18, 32), 3: (20, 32), 6: (22, 32), 7: (24, 32), 8: (34, 32), 9: (36, 32),
    10: (84, 256), 11: (110, 256), 12: (144, 256), 13: (176, 256), 14: (210, 256), 15: (292, 256),
}

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STR, _ARR = 8, 9


class GGUFError(ValueError):
    pass


class _Reader:
    def __init__(self, buf):
        self.buf, self.off = buf, 0

    def take(self, fmt):
        try:
            v = struct.unpack_from(fmt, self.buf, self.off)[0]
        except struct.error as e:
            raise GGUFError(f"file ends inside the header ({e})") from None
        self.off += struct.calcsize(fmt)
        return v

    def string(self):
        n = self.take("<Q")
        if self.off + n > len(self.buf):
            raise GGUFError("string runs past the end of the file")
        s = bytes(self.buf[self.off:self.off + n]).decode("utf-8", "replace")
        self.off += n
        return s

    def value(self, typ):
        if typ in _SCALAR:
            return self.take(_SCALAR[typ])
        if typ == _STR:
            return self.string()
        if typ == _ARR:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise GGUFError(f"unknown metadata type {typ}")


def tensor_nbytes(ggml_type, dims):
    if ggml_type not in BLOCK:
        raise GGUFError(f"unknown GGML type {ggml_type}")
    bb, be = BLOCK[ggml_type]
    n = int(np.prod(dims, dtype=np.int64)) if dims else 1
    if n % be:
        raise GGUFError(f"{n} elements is not a whole number of type-{ggml_type} blocks")
    return n // be * bb


def read(path):
    """-> (metadata dict, {name: (ggml_type, dims, uint8 bytes)})."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    r = _Reader(mm)
    magic, version = r.take("<I"), r.take("<I")
    if magic != 0x46554747:
        raise GGUFError("not a GGUF file")
    if version != 3:
        raise GGUFError(f"GGUF version {version} (3 expected)")
    n_tensors, n_kv = r.take("<Q"), r.take("<Q")
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        meta[key] = r.value(r.take("<I"))
    infos = []
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("<I")
        dims = [r.take("<Q") for _ in range(nd)]
        typ, off = r.take("<I"), r.take("<Q")
        infos.append((name, dims, typ, off))
    align = int(meta.get("general.alignment", 32))
    base = (r.off + align - 1) // align * align
    tensors = {}
    for name, dims, typ, off in infos:
        nb = tensor_nbytes(typ, dims)
        start = base + off
        if start + nb > len(mm):
            raise GGUFError(f"tensor {name} runs past the end of the file")
        tensors[name] = (typ, dims, mm[start:start + nb])
    return meta, tensors


def arch_detect(meta, tensors):
    """The llama.* hyper-parameters, with pickle_arch_detect's defaults."""
    def get(k, d):
        return meta.get("llama." + k, d)
    a = {
        "n_layers": int(get("block_count", -1)),
        "hidden_dim": int(get("embedding_length", -1)),
        "intermediate_dim": int(get("feed_forward_length", -1)),
        "n_heads": int(get("attention.head_count", -1)),
        "max_seq": int(get("context_length", 2048)),
        "rms_eps": float(get("attention.layer_norm_rms_epsilon", 1e-5)),
        "rope_theta": float(get("rope.freq_base", 10000.0)),
        "tie_word_embeddings": int(get("tie_word_embeddings", 0)),
    }
    a["n_kv_heads"] = int(get("attention.head_count_kv", a["n_heads"]))
    rope_dim = int(get("rope.dimension_count", 0))
    a["head_dim"] = rope_dim if rope_dim else (a["hidden_dim"] // a["n_heads"] if a["n_heads"] > 0 else -1)
    vs = int(get("vocab_size", -1))
    if vs <= 0:
        if "token_embd.weight" not in tensors or not tensors["token_embd.weight"][1]:
            raise GGUFError("no vocab size and no token_embd.weight")
        vs = int(tensors["token_embd.weight"][1][-1])
    a["vocab_size"] = vs
    if min(a["n_layers"], a["hidden_dim"], a["n_heads"], a["intermediate_dim"], a["vocab_size"]) <= 0:
        raise GGUFError("missing llama.* hyper-parameters")
    return a
