"""KV-cache slot manager for continuously batched decode.

The reference serves one conversation at a time: pickle_chat_loop allocates a
KV cache per call and decodes a single sequence (src/pickle_host.c:433-521).
A server instead keeps many requests in flight, each at its own position, and
admits new requests as others finish. KVSlots does that bookkeeping over the
n_seqs cache slots of one PickleCuda handle:

  * admit(req) takes a free slot (the slot's old rows are simply
    overwritten, because a request only attends rows below its own position);
  * prefill(req, layer, q, k, v, ao) runs the request's prompt into its slot
    (pickle_cuda_prefill_slot_dev) - call it for every layer, then
    advance(req, T);
  * decode(layer, reqs, q, k, v, ao) runs one decode step of several
    requests at once, each at its own position in its own slot
    (pickle_cuda_decode_ragged_dev) - call it for every layer, then
    advance(reqs);
  * release(req) returns the slot.

Positions live on the host; the device copies of the (position, slot)
arrays of a batch are rebuilt when the batch or the positions change. They
are made on the stream the decode runs on, and marked as used there, so
the caching allocator does not hand their memory to another tensor while
a decode on that stream may still read it.
"""


class SlotError(RuntimeError):
    pass


class KVSlots:
    def __init__(self, cu):
        self.cu = cu
        self.free = list(range(cu.n_seqs - 1, -1, -1))
        self.slot_of = {}
        self.pos = {}
        self._batch_key = None
        self._dev = None

    def admit(self, req):
        if req in self.slot_of:
            raise SlotError(f"request {req!r} already holds slot {self.slot_of[req]}")
        if not self.free:
            raise SlotError("no free KV slot")
        s = self.free.pop()
        self.slot_of[req] = s
        self.pos[req] = 0
        return s

    def release(self, req):
        s = self.slot_of.pop(req)
        del self.pos[req]
        self.free.append(s)
        self._batch_key = None

    def position(self, req):
        return self.pos[req]

    def advance(self, reqs, n=1):
        if not isinstance(reqs, (list, tuple)):
            reqs = [reqs]
        for r in reqs:
            if self.pos[r] + n > self.cu.max_seq:
                raise SlotError(f"request {r!r} would pass max_seq")
            self.pos[r] += n
        self._batch_key = None

    def prefill(self, req, layer, q, k, v, ao, precision=None, stream=None):
        """Prompt rows [pos, pos + T) of `req` (q [T][H][D], k/v [T][HK][D])."""
        from .api import PREFILL_F32
        T = q.shape[0]
        self.cu.prefill_slot_dev(layer, self.slot_of[req], self.pos[req], T, q, k, v, ao,
                                 PREFILL_F32 if precision is None else precision, stream)

    def batch_arrays(self, reqs, stream=None):
        """Device int32 (positions, slots) of `reqs` and the largest position,
        made on `stream` (a torch.cuda.Stream; torch's current stream otherwise)."""
        import torch
        key = tuple(reqs)
        if key != self._batch_key:
            pos = [self.pos[r] for r in reqs]
            slots = [self.slot_of[r] for r in reqs]
            dev = torch.device("cuda", self.cu.device)
            st = stream if isinstance(stream, torch.cuda.Stream) else torch.cuda.current_stream(dev)
            with torch.cuda.stream(st):
                p = torch.tensor(pos, dtype=torch.int32, device=dev)
                s = torch.tensor(slots, dtype=torch.int32, device=dev)
            self._dev = (p, s, max(pos))
            self._batch_key = key
        if isinstance(stream, torch.cuda.Stream):
            # A batch made on another stream is also read on this one.
            self._dev[0].record_stream(stream)
            self._dev[1].record_stream(stream)
        return self._dev

    def decode(self, layer, reqs, q, k, v, ao, stream=None):
        """One decode step of `reqs` (q [n][H][D], k/v [n][HK][D], ao [n][H][D])."""
        pos, slots, max_pos = self.batch_arrays(reqs, stream)
        if max_pos >= self.cu.max_seq:
            raise SlotError("a request is at max_seq")
        self.cu.decode_ragged_dev(layer, pos, q, k, v, ao, slots=slots, max_pos=max_pos, stream=stream)
