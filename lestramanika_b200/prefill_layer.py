"""The attention half of one layer for a whole prompt, on the device.

The reference's prefill runs its forward once per prompt token: for every
token it projects the normed activation to q, k and v
(pickle_fast_matmul_dispatch, src/pickle_fast.c:1903-1907), runs the
attention block for that position (:1910-2094: RoPE, cache append, softmax
over the keys so far) and projects the block's output (:2112). LayerPrefill
does the same for all T tokens at once:

  q, k, v = x Wq^T, x Wk^T, x Wv^T     pickle_cuda_matmul_dev (tensor-core GEMM
                                       over the raw GGML weight blocks)
  ao      = attention(q, k, v)         pickle_cuda_prefill_dev (RoPE, append to
                                       the device KV cache, causal attention)
  out     = ao Wo^T                    pickle_cuda_matmul_dev

Every intermediate stays on the device. The weights are raw GGML bytes in
device memory, given as (ggml_type, uint8 tensor), with each matrix
[out][in] as the reference stores it. The GEMM's workspace is allocated
once, at construction, for the largest prompt.
"""
import torch

from . import api


class LayerPrefill:
    def __init__(self, cu, wq, wk, wv, wo, hidden, max_tokens):
        """cu: the PickleCuda handle whose KV cache the prompt fills; wq / wk /
        wv / wo: (ggml_type, device uint8 tensor) of [H*D][hidden],
        [HK*D][hidden], [HK*D][hidden] and [hidden][H*D]; max_tokens: the
        longest prompt run() will be given."""
        self.cu, self.hidden, self.max_tokens = cu, hidden, max_tokens
        self.qd, self.kd = cu.H * cu.D, cu.HK * cu.D
        self.w = {"q": wq, "k": wk, "v": wv, "o": wo}
        dev = torch.device("cuda", cu.device)
        ws = max(api.matmul_workspace(self.qd, hidden, max_tokens), api.matmul_workspace(self.kd, hidden, max_tokens),
                 api.matmul_workspace(hidden, self.qd, max_tokens))
        self.ws = torch.empty(ws, dtype=torch.uint8, device=dev)
        self.q = torch.empty((max_tokens, self.qd), device=dev)
        self.k = torch.empty((max_tokens, self.kd), device=dev)
        self.v = torch.empty((max_tokens, self.kd), device=dev)
        self.ao = torch.empty((max_tokens, self.qd), device=dev)

    def _mm(self, which, x, y, out_n, in_n, T, stream):
        t, W = self.w[which]
        api.matmul_dev(t, W, out_n, in_n, x, y, T, workspace=self.ws, stream=stream)

    def run(self, layer, pos0, xn, out, precision=api.PREFILL_BF16, stream=None):
        """Positions [pos0, pos0 + T) of sequence 0: xn [T][hidden] (the
        normed input, f32, device) -> out [T][hidden] (the attention output
        projection, before the residual add). The rotated k and v of the
        prompt are appended to the cache of `layer`."""
        T = xn.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"prompt of {T} tokens > max_tokens {self.max_tokens}")
        q, k, v, ao = self.q[:T], self.k[:T], self.v[:T], self.ao[:T]
        self._mm("q", xn, q, self.qd, self.hidden, T, stream)
        self._mm("k", xn, k, self.kd, self.hidden, T, stream)
        self._mm("v", xn, v, self.kd, self.hidden, T, stream)
        self.cu.prefill_dev(layer, 1, pos0, T, q, k, v, ao, precision, stream)
        self._mm("o", ao, out, self.hidden, self.qd, T, stream)
        return out
