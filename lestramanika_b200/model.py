"""A Llama-family GGUF model whose whole forward pass runs on the device.

Host-side mirror of pickle_fast_state_init / pickle_fast_forward and of the
greedy loop of pickle_chat_loop (lee-muriithi-kingori/lestramanika
src/pickle_fast.c:1497-1662, 1822-2184; src/pickle_host.c:473-521) over the
C ABI's pickle_cuda_model_* entry points. Tensors are found by the names the
reference looks up (src/pickle_fast.c:1530-1633); missing ones raise
PICKLE_ERR_ARCH like the reference. Every weight goes to the device in its
raw GGML blocks; a quantized token embedding becomes an F32 table on the
device at load, as pickle_fast_state_init makes one (:1551-1584).
"""
import ctypes

import numpy as np

from . import api, gguf

LAYER_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
               "ffn_down")


def _host_tensor(typ, data):
    a = np.ascontiguousarray(np.asarray(data).view(np.uint8).reshape(-1))
    return api.Tensor(int(typ), a.ctypes.data, a.nbytes), a


def _dev_tensor(typ, t):
    return api.Tensor(int(typ), t.data_ptr(), t.numel() * t.element_size()), t


class PickleModel:
    def __init__(self, tensors, arch, device=0, max_tokens=512, precision=api.PREFILL_F32, rope_inv_freq=None,
                 n_seqs=1):
        """tensors: {gguf name: (ggml_type, data)} with data a numpy array of the
        raw bytes (host) or a torch CUDA tensor (used in place, kept alive by
        this object); arch: the dict gguf.arch_detect returns; n_seqs: cache
        slots, for generate_batch / forward_batch_dev."""
        self.arch = dict(arch)
        self.VS, self.max_seq = arch["vocab_size"], arch["max_seq"]
        keep = []
        on_dev = None

        def tensor(name, required=True):
            nonlocal on_dev
            if name not in tensors:
                if required:
                    raise api.PickleError(-8, "model", f"missing tensor {name}")
                return api.Tensor(0, None, 0)
            typ, data = tensors[name]
            dev = hasattr(data, "data_ptr")
            if on_dev is None:
                on_dev = dev
            elif on_dev != dev:
                raise ValueError("tensors must be all on the host or all on the device")
            t, owner = _dev_tensor(typ, data) if dev else _host_tensor(typ, data)
            keep.append(owner)
            return t

        p = api.ModelParams()
        for k in ("n_layers", "hidden_dim", "intermediate_dim", "n_heads", "n_kv_heads", "head_dim", "vocab_size",
                  "max_seq"):
            setattr(p, k, int(arch[k]))
        p.rms_eps, p.rope_theta = float(arch["rms_eps"]), float(arch["rope_theta"])
        if rope_inv_freq is not None:
            self._inv = np.ascontiguousarray(rope_inv_freq, np.float32)
            p.rope_inv_freq = self._inv.ctypes.data_as(api._fp)
        p.max_tokens, p.prefill_precision = int(max_tokens), int(precision)
        p.token_embd = tensor("token_embd.weight")
        p.output_norm = tensor("output_norm.weight", required=False)
        # Tied embeddings, or no output.weight: the lm_head is token_embd
        # (src/pickle_fast.c:2142).
        p.output = api.Tensor(0, None, 0) if arch.get("tie_word_embeddings") else tensor("output.weight", False)
        nl = int(arch["n_layers"])
        layers = (api.Tensor * (nl * api.LAYER_TENSORS))()
        for L in range(nl):
            for j, n in enumerate(LAYER_NAMES):
                layers[L * api.LAYER_TENSORS + j] = tensor(f"blk.{L}.{n}.weight")
        p.layers = layers
        p.weights_on_device = 1 if on_dev else 0
        p.n_seqs = int(n_seqs)
        self.n_seqs = max(1, int(n_seqs))
        h = ctypes.c_void_p()
        rc = api.lib().pickle_cuda_model_load(ctypes.byref(p), int(device), ctypes.byref(h))
        if rc != 0:
            raise api.PickleError(rc, "pickle_cuda_model_load")
        self._h = h
        self._keep = keep if on_dev else None   # host copies are uploaded at load
        self.device = device

    @classmethod
    def from_gguf(cls, path, device=0, **kw):
        meta, t = gguf.read(path)
        arch = gguf.arch_detect(meta, t)
        tensors = {name: (typ, data) for name, (typ, dims, data) in t.items()}
        return cls(tensors, arch, device=device, **kw)

    def _check(self, rc, what):
        if rc != 0:
            detail = api.lib().pickle_cuda_model_last_error(self._h)
            raise api.PickleError(rc, what, detail.decode() if detail else "")

    def close(self):
        if getattr(self, "_h", None):
            api.lib().pickle_cuda_model_free(self._h)
            self._h = None
            self._keep = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, kv_pos):
        """pickle_fast_forward: -> (logits of the last token [vocab], new kv_pos)."""
        tok = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.VS, np.float32)
        pos = ctypes.c_size_t(int(kv_pos))
        self._check(api.lib().pickle_cuda_forward(self._h, tok.ctypes.data_as(api._i32p), tok.size,
                                                  logits.ctypes.data_as(api._fp), ctypes.byref(pos)),
                    "pickle_cuda_forward")
        return logits, pos.value

    def forward_slot(self, slot, tokens, kv_pos):
        """pickle_fast_forward for the sequence in cache slot `slot`."""
        tok = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.VS, np.float32)
        pos = ctypes.c_size_t(int(kv_pos))
        self._check(api.lib().pickle_cuda_forward_slot(self._h, int(slot), tok.ctypes.data_as(api._i32p), tok.size,
                                                       logits.ctypes.data_as(api._fp), ctypes.byref(pos)),
                    "pickle_cuda_forward_slot")
        return logits, pos.value

    def forward_batch_dev(self, tokens_dev, pos_dev, slot_dev, max_pos, logits_dev, next_dev=None, stream=None):
        """One decode step of n sequences (device int32 tokens / positions /
        slots [n], f32 logits [n][vocab], optional int32 argmax ids [n])."""
        self._check(api.lib().pickle_cuda_forward_batch_dev(self._h, tokens_dev.numel(), api._ptr(tokens_dev),
                                                            api._ptr(pos_dev), api._ptr(slot_dev), int(max_pos),
                                                            api._ptr(logits_dev), api._ptr(next_dev),
                                                            api._stream(stream)), "pickle_cuda_forward_batch_dev")

    def generate_batch(self, prompts, n_gen, eos_id=-1):
        """Greedy generation of many requests with continuous batching: up to
        n_seqs requests hold a cache slot each; every step decodes all of them
        together (forward_batch_dev); a finished request frees its slot and
        the next waiting prompt is admitted (its prompt runs into that slot,
        forward_slot). Each request's ids are those generate(prompt, n_gen,
        eos_id) gives. -> list of id arrays, in the order of prompts."""
        import torch
        dev = self._torch_device()
        waiting = list(range(len(prompts)))[::-1]
        free = list(range(self.n_seqs))[::-1]
        ids = [[] for _ in prompts]
        slot, pos, cur = {}, {}, {}
        active = []

        def done(r):
            return (len(ids[r]) >= n_gen or (eos_id >= 0 and ids[r][-1] == eos_id) or pos[r] >= self.max_seq)

        def admit():
            while waiting and free:
                r = waiting.pop()
                if n_gen <= 0:
                    continue
                s = free.pop()
                logits, p = self.forward_slot(s, prompts[r], 0)
                slot[r], pos[r] = s, p
                ids[r].append(int(np.argmax(logits)))
                if done(r):
                    free.append(s)
                else:
                    active.append(r)

        logits_dev = torch.empty((self.n_seqs, self.VS), device=dev)
        next_dev = torch.empty(self.n_seqs, dtype=torch.int32, device=dev)
        admit()
        while active:
            n = len(active)
            host = np.array([[ids[r][-1] for r in active], [pos[r] for r in active], [slot[r] for r in active]],
                            np.int32)
            d = torch.from_numpy(host).to(dev)
            self.forward_batch_dev(d[0], d[1], d[2], int(host[1].max()), logits_dev[:n], next_dev[:n])
            nxt = next_dev[:n].cpu().numpy()
            self.sync()
            still = []
            for r, t in zip(active, nxt):
                pos[r] += 1
                ids[r].append(int(t))
                if done(r):
                    free.append(slot[r])
                else:
                    still.append(r)
            active[:] = still
            admit()
        return [np.array(x, np.int32) for x in ids]

    def _torch_device(self):
        import torch
        return torch.device("cuda", self.device)

    def forward_dev(self, tokens_dev, pos0, logits_dev, next_dev=None, stream=None):
        """Asynchronous forward on device buffers (int32 tokens, f32 logits [vocab])."""
        self._check(api.lib().pickle_cuda_forward_dev(self._h, api._ptr(tokens_dev), tokens_dev.numel(), int(pos0),
                                                      api._ptr(logits_dev), api._ptr(next_dev),
                                                      api._stream(stream)), "pickle_cuda_forward_dev")

    def sync(self, stream=None):
        self._check(api.lib().pickle_cuda_model_sync(self._h, api._stream(stream)), "pickle_cuda_model_sync")

    def generate(self, prompt, n_gen, eos_id=-1, kv_pos=0, want_logits=True, temp=0.0, top_p=0.0, seed=0):
        """The decode loop of pickle_chat_loop -> (ids, last logits, kv_pos):
        greedy when temp <= 0, else pickle_fast_sample_temp with seed + i."""
        tok = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(n_gen, 1), np.int32)
        n_out = ctypes.c_int(0)
        logits = np.empty(self.VS, np.float32) if want_logits else None
        pos = ctypes.c_size_t(int(kv_pos))
        self._check(api.lib().pickle_cuda_generate_sampled(
            self._h, tok.ctypes.data_as(api._i32p), tok.size, int(n_gen), int(eos_id), float(temp), float(top_p),
            int(seed) & 0xFFFFFFFF, ids.ctypes.data_as(api._i32p), ctypes.byref(n_out),
            logits.ctypes.data_as(api._fp) if logits is not None else None, ctypes.byref(pos)),
            "pickle_cuda_generate_sampled")
        return ids[:n_out.value].copy(), logits, pos.value
