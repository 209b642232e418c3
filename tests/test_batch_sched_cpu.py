"""The continuous-batching loop of PickleModel.generate_batch, on the CPU:
the model's device calls are replaced by a deterministic fake (the next id
is a function of the last id and its position), so the test checks the
scheduling itself - admission into free slots, one batched step for all
active requests, retirement after n_gen ids, after the eos id or at a full
cache, and the next waiting prompt taking the freed slot - against a plain
per-request loop with the chat loop's rules."""
import numpy as np
import torch

from lestramanika_b200.model import PickleModel

V = 97


def _next(tok, pos):
    return (tok * 31 + pos * 7 + 3) % V


class FakeModel(PickleModel):
    def __init__(self, n_seqs, max_seq):
        self.n_seqs, self.max_seq, self.VS, self.device = n_seqs, max_seq, V, 0
        self.slot_pos = {}          # slot -> the position its next token must take
        self.max_active = 0

    def _torch_device(self):
        return torch.device("cpu")

    def forward_slot(self, slot, tokens, kv_pos):
        assert 0 <= slot < self.n_seqs and kv_pos == 0
        pos = kv_pos + len(tokens)
        self.slot_pos[slot] = pos
        logits = np.zeros(V, np.float32)
        logits[_next(tokens[-1], pos - 1)] = 1.0
        return logits, pos

    def forward_batch_dev(self, tokens_dev, pos_dev, slot_dev, max_pos, logits_dev, next_dev=None, stream=None):
        n = tokens_dev.numel()
        self.max_active = max(self.max_active, n)
        assert n <= self.n_seqs and len(set(slot_dev.tolist())) == n
        assert int(pos_dev.max()) == max_pos < self.max_seq
        for i in range(n):
            s, p = int(slot_dev[i]), int(pos_dev[i])
            assert self.slot_pos.get(s) == p, "a slot's positions must follow on (one request per slot)"
            self.slot_pos[s] = p + 1
            next_dev[i] = _next(int(tokens_dev[i]), p)

    def sync(self, stream=None):
        pass

    def close(self):
        pass


def _single(prompt, n_gen, eos_id, max_seq):
    """pickle_chat_loop's rules for one request with the fake model."""
    ids, pos = [], len(prompt)
    cur = _next(prompt[-1], pos - 1)
    while True:
        ids.append(cur)
        if len(ids) >= n_gen or cur == eos_id or pos >= max_seq:
            return ids
        cur = _next(cur, pos)
        pos += 1


def _run(n_seqs, n_req, n_gen, eos_id, max_seq, seed):
    rng = np.random.default_rng(seed)
    prompts = [[int(t) for t in rng.integers(0, V, size=int(rng.integers(1, 9)))] for _ in range(n_req)]
    m = FakeModel(n_seqs, max_seq)
    got = PickleModel.generate_batch(m, prompts, n_gen, eos_id=eos_id)
    want = [_single(p, n_gen, eos_id, max_seq) for p in prompts]
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)
    return m


def test_more_requests_than_slots():
    m = _run(n_seqs=3, n_req=8, n_gen=12, eos_id=-1, max_seq=64, seed=1)
    assert m.max_active == 3


def test_eos_and_full_cache_retire_early():
    _run(n_seqs=2, n_req=6, n_gen=40, eos_id=5, max_seq=64, seed=2)
    _run(n_seqs=4, n_req=5, n_gen=40, eos_id=-1, max_seq=14, seed=3)   # prompts of up to 8: the cache fills


def test_one_id_per_request_needs_no_step():
    m = _run(n_seqs=2, n_req=4, n_gen=1, eos_id=-1, max_seq=64, seed=4)
    assert m.max_active == 0
