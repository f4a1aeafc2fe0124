"""Host models of the streaming kernel's work schedules
(quickruncuda_b200/csrc/side_aware_b200.cu).  Queue schedule (SideWalk): the
queue-position -> pair interleave must be a bijection for every size, and any
split of the positions into grabs, on both sides, must read every byte exactly
once whatever the side map says.  Balanced schedule (read_share + read_tail):
static blocks plus queued tail blocks, with stealing, cover every chunk once.  The device code itself is checked on the GPU by the checked build
(tests/test_absmax_gpu.py::test_checked_build_every_byte_once_in_bounds)."""
import numpy as np
import pytest


def pair_of(c, npairs, stride_log2=11, grab_log2=3):
    """Same arithmetic as SideWalk::pair_of."""
    if stride_log2 == 0:
        return c
    g1 = (1 << grab_log2) - 1
    block_log2 = stride_log2 + grab_log2
    main = (npairs >> block_log2) << block_log2
    tail_stride = (npairs - main) >> grab_log2
    if c < main:
        r = c & ((1 << block_log2) - 1)
        return (c - r) + ((r & g1) << stride_log2) + (r >> grab_log2)
    r = c - main
    if r < (tail_stride << grab_log2):
        return main + (r & g1) * tail_stride + (r >> grab_log2)
    return c


@pytest.mark.parametrize("npairs", [0, 1, 7, 8, 9, 100, 2047, 2048, 16383, 16384, 16385, 40000, 488281])
@pytest.mark.parametrize("stride_log2,grab_log2", [(11, 3), (4, 2), (0, 3), (6, 0), (11, 4)])
def test_interleave_is_a_bijection(npairs, stride_log2, grab_log2):
    seen = np.zeros(npairs, dtype=np.int8)
    for c in range(npairs):
        p = pair_of(c, npairs, stride_log2, grab_log2)
        assert 0 <= p < npairs
        seen[p] += 1
    assert np.all(seen == 1)


def test_aligned_grab_spreads_and_neighbours_are_adjacent():
    n = 5 * 16384 + 1234
    grab = [pair_of(c, n) for c in range(16, 24)]           # one 8-position grab
    assert np.all(np.diff(grab) == 2048)
    firsts = [pair_of(c, n) for c in range(0, 64, 8)]       # first pair of 8 consecutive grabs
    assert np.all(np.diff(firsts) == 1)


def test_two_sides_cover_every_byte_once(oracle):
    """Side 0 reads, for each pair, the half homed on side 0 and side 1 the
    other half, for any mask / page bits and any grab split."""
    rng = np.random.default_rng(0)
    C = 4096
    for trial in range(20):
        npairs = int(rng.integers(1, 3000))
        base = int(rng.integers(0, 1 << 30)) & ~(2 * C - 1)
        mask = (int(rng.integers(0, 1 << 21)) & ~0xFFF) | 0x1000
        page_bits = rng.integers(0, 2, size=(npairs * 2 * C >> 21) + 2)
        covered = np.zeros(2 * npairs, dtype=np.int8)          # chunk granularity
        for side in (0, 1):
            c = 0
            while c < npairs:                                    # random grab sizes
                size = int(rng.integers(1, 9))
                for q in range(c, min(c + size, npairs)):
                    p = pair_of(q, npairs)
                    addr = base + p * 2 * C
                    pb = int(page_bits[(addr - (base & ~((1 << 21) - 1))) >> 21])
                    half = oracle.pair_half(addr, mask, pb, side)
                    covered[2 * p + half] += 1
                c += size
        assert np.all(covered == 1), trial


def _balanced_cover(oracle, npairs, k0, k1, groups_per_cta, eighths, rng):
    """Host model of the balanced schedule (reduce_run with static shares plus
    read_tail): side s has K_s SMs of G groups; 8-pair block b < R/8 belongs
    to group b mod (K_s * G); blocks past R are claimed from the side's queue
    in any order, and a group whose queue is empty claims from the other
    side's queue, reading that side's chunks."""
    C = 4096
    base = 1 << 30
    mask = 0x1EF000
    page_bits = rng.integers(0, 2, size=(npairs * 2 * C >> 21) + 2)
    R = (npairs * eighths // 8) & ~7
    covered = np.zeros(2 * npairs, dtype=np.int8)

    def read_pair(p, side):
        addr = base + p * 2 * C
        half = oracle.pair_half(addr, mask, int(page_bits[(addr - base) >> 21]), side)
        covered[2 * p + half] += 1

    for side, k in ((0, k0), (1, k1)):
        groups = k * groups_per_cta
        for g in range(groups):
            b = g
            while b * 8 < R:
                for p in range(b * 8, min(b * 8 + 8, R)):
                    read_pair(p, side)
                b += groups
    nb = (npairs - R + 7) // 8
    counters = [0, 0]
    # claims in a random interleaving of groups from both sides, each group
    # draining its own queue then the other one
    agents = [(s, False) for s in (0, 1) for _ in range(3)]
    while agents:
        i = int(rng.integers(0, len(agents)))
        side, stolen = agents[i]
        q = side ^ 1 if stolen else side
        c = counters[q]
        counters[q] += 1
        if c >= nb:
            if stolen:
                agents.pop(i)
            else:
                agents[i] = (side, True)
            continue
        for p in range(R + 8 * c, min(R + 8 * c + 8, npairs)):
            read_pair(p, q)
    return covered


@pytest.mark.parametrize("npairs,k0,k1", [(1, 74, 74), (7, 70, 78), (100, 74, 74), (2047, 70, 78),
                                          (5000, 76, 72), (12345, 1, 3)])
@pytest.mark.parametrize("eighths", [5, 7, 8])
def test_balanced_schedule_covers_every_chunk_once(oracle, npairs, k0, k1, eighths):
    rng = np.random.default_rng(npairs + eighths)
    covered = _balanced_cover(oracle, npairs, k0, k1, 4, eighths, rng)
    assert np.all(covered == 1)


def _first_block(sm_first, K, G, k, g):
    """Same arithmetic as Shares::first_block."""
    return g * K + k if sm_first else k * G + g


@pytest.mark.parametrize("K", [1, 3, 70, 74, 78])
@pytest.mark.parametrize("G", [1, 2, 4])
@pytest.mark.parametrize("sm_first", [False, True])
def test_share_groups_are_a_bijection_and_sm_first_balances(K, G, sm_first):
    """Every (SM k, group g) pair starts at a distinct block of [0, K*G), so
    blocks b, b + K*G, ... cover every block once; with the SM-first order
    the blocks per SM differ by at most one for every input size."""
    firsts = sorted(_first_block(sm_first, K, G, k, g) for k in range(K) for g in range(G))
    assert firsts == list(range(K * G))
    for nb in (0, 1, 5, 64, K * G - 1, K * G, K * G + 3, 1024, 4096 + 7):
        per_sm = [sum(len(range(_first_block(sm_first, K, G, k, g), nb, K * G)) for g in range(G))
                  for k in range(K)]
        assert sum(per_sm) == nb
        assert max(per_sm) - min(per_sm) <= (1 if sm_first else G)
