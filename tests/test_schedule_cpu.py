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


SUBQUEUES = 4


def schedule_chunks(npairs, warps, rng):
    """Chunk indices (2*pair + half) read by the walk, as SideWalk does it:
    the static round hands chunk h to global warp h for the first
    min(npairs, warps/2) pairs; the rest is split into SUBQUEUES slices per
    side, each taken in random grab sizes and mapped through pair_of().
    Returns (side, chunk) for every chunk read; `half` for queued pairs is
    the oracle's choice for that side."""
    nstatic = min(npairs, warps // 2)
    out = [(None, h) for h in range(2 * nstatic)]
    queued = npairs - nstatic
    for side in (0, 1):
        for k in range(SUBQUEUES):
            first = queued * k // SUBQUEUES
            size = queued * (k + 1) // SUBQUEUES - first
            c = 0
            while c < size:
                g = int(rng.integers(1, 9))
                for q in range(c, min(c + g, size)):
                    out.append((side, nstatic + first + pair_of(q, size)))
                c += g
    return out, nstatic


@pytest.mark.parametrize("npairs", [1, 5, 100, 2368, 2369, 5000, 40000])
def test_static_round_and_slices_cover_every_byte_once(oracle, npairs):
    """Any mask / page bits and any grab split: every chunk exactly once."""
    rng = np.random.default_rng(npairs)
    C = 4096
    warps = 4736
    base = int(rng.integers(0, 1 << 30)) & ~(2 * C - 1)
    mask = (int(rng.integers(0, 1 << 21)) & ~0xFFF) | 0x1000
    page_bits = rng.integers(0, 2, size=(npairs * 2 * C >> 21) + 2)
    covered = np.zeros(2 * npairs, dtype=np.int32)
    reads, nstatic = schedule_chunks(npairs, warps, rng)
    for side, x in reads:
        if side is None:                      # static round: chunk index given directly
            covered[x] += 1
            continue
        p = x
        addr = base + p * 2 * C
        pb = int(page_bits[(addr - (base & ~((1 << 21) - 1))) >> 21])
        covered[2 * p + oracle.pair_half(addr, mask, pb, side)] += 1
    assert np.all(covered == 1)
