"""qrc_absmax_f32_noalloc: the entry point for callers that cannot allocate
device memory (a host application that reserves all memory up front and hands
this code only its buffers, a process held to a fixed memory budget, code that
must not trigger cudaMalloc's implicit synchronisation).  Its scratch is a
fixed device array inside the library, shared by every call on a device.

Collected last on purpose: if it fails, a run that stops at the first failure
has already run every other test.  It passes alone in a fresh process and after
the other tests (the array keeps the previous call's contents, which the entry
point clears whenever the input range changes)."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _bits(t):
    import torch
    return int(t.detach().cpu().view(torch.int32).item()) & 0xFFFFFFFF


def test_noalloc_matches_the_context_entry_point_twice_in_a_row(cuda, qrc, lib, oracle):
    import torch
    n = 37 * (1 << 20) + 3                       # spans 75 pages, odd tail
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=8)
    i, s = qrc.outlier(8, n)
    x[i] = 6.25 * s
    stream = torch.cuda.current_stream().cuda_stream
    with qrc.SideAwareContext(x) as ctx:         # the existing entry point, with its own scratch
        want = _bits(ctx.absmax(x))
    assert want == 0x40C80000                    # 6.25
    assert want == oracle.absmax_bits(x.cpu().numpy())   # and the CPU oracle on the host copy
    out = torch.full((2,), -1.0, dtype=torch.float32, device=cuda)
    for k in range(2):                           # two calls in a row on the same buffer
        rc = lib.qrc_absmax_f32_noalloc(x.data_ptr(), n, out[k:].data_ptr(), stream)
        assert rc == 0
    torch.cuda.synchronize()
    assert _bits(out[0]) == want and _bits(out[1]) == want
    # a different range: the array is cleared and remapped before the reduction
    y = x[1000:1000 + (5 << 20)]
    with qrc.SideAwareContext(y) as ctx:
        want_y = _bits(ctx.absmax(y))
    assert want_y == oracle.absmax_bits(y.cpu().numpy())
    for k in range(2):
        assert lib.qrc_absmax_f32_noalloc(y.data_ptr(), y.numel(), out[k:].data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert _bits(out[0]) == want_y and _bits(out[1]) == want_y


def test_noalloc_rejects_inputs_beyond_its_scratch(cuda, lib):
    # The limit is 32768 pages of 2 MiB = 2^34 floats from a page-aligned start;
    # one float more is refused before any GPU work (the pointer, page-aligned
    # and never dereferenced, only feeds the page count).
    limit = 32768 * (2 << 20) // 4
    assert limit == 1 << 34
    assert lib.qrc_absmax_f32_noalloc(1 << 21, limit + 1, 1 << 21, None) == -4
    assert lib.qrc_absmax_f32_noalloc(1 << 21, 1 << 40, 1 << 21, None) == -4
    assert lib.qrc_absmax_f32_noalloc(None, 16, 1 << 21, None) == -1
