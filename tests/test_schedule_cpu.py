"""Host model of the streaming kernel's work schedule (SideWalk in
quickruncuda_b200/csrc/side_aware_b200.cu): the queue-position -> pair
interleave must be a bijection for every size, and any split of the positions
into grabs, on both sides, must read every byte exactly once whatever the side
map says.  The device code itself is checked on the GPU by the checked build
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
