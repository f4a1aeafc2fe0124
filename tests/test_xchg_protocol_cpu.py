"""Host model of the in-kernel cross-GPU exchange (xchg_max_u32 in
quickruncuda_b200/csrc/side_aware_b200.cu): each rank, at the end of launch
e, stores (e, value) into slot [e mod 2][rank] of every rank's array, then
waits until its own array holds epoch e in every slot of parity e mod 2.

The model runs N ranks as interleaved steps under random scheduling. It
checks two things: every rank's launch e combines exactly the values that
the ranks published for e (a slot is never overwritten by epoch e + 2 before
its owner has read epoch e), and no rank waits forever."""
import random

import pytest


def _simulate(world, launches, seed):
    rng = random.Random(seed)
    slots = [[[(0, 0)] * world for _ in range(2)] for _ in range(world)]      # slots[owner][parity][writer]
    value = lambda r, e: (e * 7919 + r * 104729) % 1000003                  # each rank's partial per launch
    state = [{"e": 1, "phase": "store", "p": 0, "q": 0, "acc": 0} for _ in range(world)]
    results = {r: [] for r in range(world)}
    steps = 0
    while any(s["e"] <= launches for s in state):
        steps += 1
        assert steps < 1_000_000, "livelock"
        r = rng.randrange(world)
        s = state[r]
        if s["e"] > launches:
            continue
        e, par = s["e"], s["e"] & 1
        if s["phase"] == "store":                       # one peer store per step
            slots[s["p"]][par][r] = (e, value(r, e))
            s["p"] += 1
            if s["p"] == world:
                s["phase"], s["q"], s["acc"] = "wait", 0, value(r, e)
        else:                                           # one poll per step
            ep, v = slots[r][par][s["q"]]
            if ep == e:
                s["acc"] = max(s["acc"], v)
                s["q"] += 1
                if s["q"] == world:
                    results[r].append(s["acc"])
                    s.update(e=e + 1, phase="store", p=0)
            else:
                assert ep < e, (r, e, s["q"], ep)      # never a newer epoch in a slot still being waited for
    for r in range(world):
        assert results[r] == [max(value(q, e) for q in range(world)) for e in range(1, launches + 1)]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("seed", range(6))
def test_epoch_parity_exchange(world, seed):
    _simulate(world, launches=25, seed=seed)
