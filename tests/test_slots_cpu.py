"""KVSlots bookkeeping (no GPU): slots are handed out and returned, positions
advance per request, and misuse is an error."""
import pytest

from lestramanika_b200.slots import KVSlots, SlotError


class _FakeHandle:
    n_seqs, max_seq, device = 3, 16, 0


def test_admit_release_reuses_slots_and_tracks_positions():
    s = KVSlots(_FakeHandle())
    a, b = s.admit("a"), s.admit("b")
    assert {a, b} == {0, 1}
    s.advance("a", 5)
    s.advance(["a", "b"])
    assert s.position("a") == 6 and s.position("b") == 1
    s.release("a")
    c = s.admit("c")
    assert c == a and s.position("c") == 0


def test_misuse_is_an_error():
    s = KVSlots(_FakeHandle())
    for r in "xyz":
        s.admit(r)
    with pytest.raises(SlotError):
        s.admit("w")                        # no free slot
    with pytest.raises(SlotError):
        s.admit("x")                        # already admitted
    with pytest.raises(SlotError):
        s.advance("x", 17)                  # past max_seq
