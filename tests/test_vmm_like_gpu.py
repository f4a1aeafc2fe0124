"""Buffers homed like an input (qrc_alloc_like) and the side-aware copy.

A context over the new buffer must find, page for page, the same die pattern
as the input's context (after lining up the two maps' side labels), and the
copy must reproduce the input bit for bit, also into ordinary memory and for
ragged ranges."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
O_SM_SIDE, O_PAGE_BITS, H_NPAGES = 256, 4096, 7


def _page_bits(m):
    n = int(m[H_NPAGES])
    return np.array([(int(m[O_PAGE_BITS + p // 32]) >> (p % 32)) & 1 for p in range(n)])


def _flip(m1, m2):
    a = m1[O_SM_SIDE:O_SM_SIDE + 256].astype(np.int64)
    b = m2[O_SM_SIDE:O_SM_SIDE + 256].astype(np.int64)
    both = (a > 0) & (b > 0)
    differ = int(np.sum(((a[both] - 1) & 1) != ((b[both] - 1) & 1)))
    return int(differ > both.sum() - differ)


@pytest.fixture(scope="module")
def src(cuda, qrc):
    import torch
    x = torch.empty(64 << 20, dtype=torch.float32, device=cuda)      # 256 MB, 128 pages
    qrc.fill_normal(x, seed=21, sigma=4.0)
    ctx = qrc.SideAwareContext(x)
    yield x, ctx
    ctx.close()


def test_alloc_like_homes_every_page_like_the_input(src, qrc):
    x, ctx = src
    y = ctx.alloc_like()
    assert y.numel() == x.numel() and y.data_ptr() % (2 << 20) == x.data_ptr() % (2 << 20)
    with qrc.SideAwareContext(y) as cy:
        assert cy.info["status"] == 0
        mx, my = ctx.read_map(), cy.read_map()
        assert np.array_equal(_page_bits(mx), _page_bits(my) ^ _flip(mx, my))


def test_side_aware_copy_is_exact(src, qrc):
    import torch
    x, ctx = src
    y = ctx.alloc_like()
    y.zero_()
    ctx.copy(x, y)
    assert torch.equal(x.view(torch.int32), y.view(torch.int32))
    z = torch.zeros_like(x)                                           # ordinary memory
    ctx.copy(x, z)
    assert torch.equal(x.view(torch.int32), z.view(torch.int32))
    for mode in (0, 1, 2):
        ctx.mode = mode
        for off, n in [(4, 8191), (1024, (1 << 22) + 12), (0, 5), (12, (64 << 20) - 12)]:
            y.zero_()
            ctx.copy(x[off:off + n], y[off:off + n])
            assert torch.equal(x[off:off + n].view(torch.int32), y[off:off + n].view(torch.int32)), (mode, off, n)
            assert int(torch.count_nonzero(y[:off])) == 0 and int(torch.count_nonzero(y[off + n:])) == 0
    ctx.mode = 0
    ctx.copy(x[3:1003], z[5:1005])                                   # unaligned: the plain copy
    assert torch.equal(x[3:1003], z[5:1005])
    lib = ctx.lib                                                    # overlap: refused; onto itself: no-op
    assert lib.qrc_copy_f32(x[0:].data_ptr(), x[8:].data_ptr(), 1000, ctx.handle, None) == -1
    assert lib.qrc_copy_f32(x[8:].data_ptr(), x[0:].data_ptr(), 1000, ctx.handle, None) == -1
    before = x[:1000].clone()
    assert lib.qrc_copy_f32(x.data_ptr(), x.data_ptr(), 1000, ctx.handle, None) == 0
    assert torch.equal(before, x[:1000])
    del y
    torch.cuda.synchronize()
