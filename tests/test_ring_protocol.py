"""CPU model of the decode kernel's shared-memory ring protocol
(lestramanika_b200/csrc/decode_splitkv.cuh): one producer lane, NSET consumer
sets of NW warps taking tiles set, set + NSET, ..., a full and an empty
mbarrier per stage, and the short-split stagger (first tile alone, the other
stages once it has landed).

An mbarrier parity wait passes when (completed phases & 1) != parity, so a
waiter more than one phase behind a barrier's true state passes early. The
model runs the protocol under random schedules and checks that every passed
wait is the intended phase: a consumer never reads a tile that has not
landed, the producer never reissues a stage whose tile is still in use, and
nothing deadlocks. Without the consumers' wait for the release of a stage's
previous tile, the hazard appears (it faulted the GPU once: a CTA finished
with a bulk copy into its shared memory still in flight)."""
import random

import pytest

K_MAX_STAGE_BYTES = 98304


def decode_cfg(D, G):
    """STAGES / NSET / NW as DecodeCfg<D, G> computes them."""
    stage_bytes = 2 * 32 * D * 4
    stages = min(max(K_MAX_STAGE_BYTES // stage_bytes, 2), 8)
    nset = max(1, min((4 if D > 128 else 8) // G, stages))
    return stages, nset, G


def _passes(completed, parity):
    return (completed & 1) != parity


def run_protocol(stages, nset, nw, n_tiles, release_wait, stagger, seed):
    rnd = random.Random(seed)
    full_done = [0] * stages            # completed phases
    empty_done = [0] * stages
    empty_arrivals = [0] * stages
    in_flight = {}                      # stage -> tile
    landed = set()
    released = set()
    p_next = 0
    # warp: [set, tile it, state] with state 0 = wait release, 1 = wait full, 2 = arrive
    warps = [[s, s, 0] for s in range(nset) for _ in range(nw)]
    for _ in range(100000):
        acts = []
        if p_next < n_tiles:
            acts.append("issue")
        if in_flight:
            acts.append("land")
        acts += [i for i, w in enumerate(warps) if w[1] < n_tiles]
        if not acts:
            return None
        a = rnd.choice(acts)
        if a == "issue":
            it = p_next
            s, u = it % stages, it // stages
            if stagger and it == 1 and not _passes(full_done[0], 0):
                continue
            if u >= 1 and not _passes(empty_done[s], (u - 1) & 1):
                continue
            if u >= 1 and (it - stages) not in released:
                return f"producer reissued stage {s} for tile {it} before tile {it - stages} was released"
            if s in in_flight:
                return f"producer reissued stage {s} while tile {in_flight[s]} is in flight"
            in_flight[s] = it
            p_next += 1
        elif a == "land":
            s = rnd.choice(sorted(in_flight))
            landed.add(in_flight.pop(s))
            full_done[s] += 1
        else:
            w = warps[a]
            it = w[1]
            s, u = it % stages, it // stages
            if w[2] == 0:
                if release_wait and nset > 1 and u >= 1 and not _passes(empty_done[s], (u - 1) & 1):
                    continue
                w[2] = 1
            elif w[2] == 1:
                if not _passes(full_done[s], u & 1):
                    continue
                if it not in landed or full_done[s] != u + 1:
                    return f"set {w[0]} passed the full wait of tile {it} (stage {s}, {full_done[s]} phases done)"
                w[2] = 2
            else:
                empty_arrivals[s] += 1
                if empty_arrivals[s] == nw:
                    empty_arrivals[s] = 0
                    empty_done[s] += 1
                    released.add(it)
                w[1] = it + nset
                w[2] = 0
    return "deadlock or livelock"


CONFIGS = sorted({decode_cfg(D, G) for D in (48, 64, 96, 128, 256) for G in (1, 2, 4, 8)})


@pytest.mark.parametrize("stages,nset,nw", CONFIGS)
def test_ring_protocol_never_passes_a_wait_early(stages, nset, nw):
    for n_tiles in (1, 2, 3, 4, 5, 7, 2 * stages, 2 * stages + 1, 17):
        stagger = n_tiles <= 2 * stages
        for seed in range(25):
            err = run_protocol(stages, nset, nw, n_tiles, True, stagger, seed)
            assert err is None, (stages, nset, nw, n_tiles, seed, err)


def test_without_the_release_wait_the_parity_hazard_appears():
    """Three stages, two sets of four warps (the GQA-4 decode): consecutive
    uses of a stage alternate between the sets, and without the release wait
    some schedule passes a full wait for a tile that has not landed."""
    failures = [run_protocol(3, 2, 4, n, False, False, seed) for n in (4, 7, 16) for seed in range(60)]
    assert any(f is not None and "passed the full wait" in f for f in failures)
