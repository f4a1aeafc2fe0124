"""The in-kernel cross-GPU maximum (qrc_absmax_f32_allreduce) on one GPU.

Two GPUs' kernels may wait on each other, but two kernels on one GPU must
not, so on one GPU the other ranks are played from the host: a test writes a
peer's (epoch, value) slot before the launch, or leaves it empty to check that
the bounded wait gives up with NaN and an error word while the context stays
usable.  The two-GPU run is tests/test_xchg_multi_gpu.py."""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
H_XCHG_ERR = 106


def _xchg(lib, rank, world):
    h = ctypes.c_void_p()
    assert lib.qrc_xchg_create(ctypes.byref(h), 0, rank, world) == 0
    return h


@pytest.fixture(scope="module")
def data(cuda, qrc):
    import torch
    x = torch.empty((1 << 22) + 3, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=12)
    x[777] = -5.5
    ctx = qrc.SideAwareContext(x)
    yield x, ctx
    ctx.close()


def test_world_of_one_equals_absmax(data):
    import torch
    x, ctx = data
    lib = ctx.lib
    h = _xchg(lib, 0, 1)
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        for i in range(5):
            assert lib.qrc_absmax_f32_allreduce(x.data_ptr(), x.numel(), out.data_ptr(), ctx.handle, h, None) == 0
            assert out.item() == 5.5
        assert lib.qrc_xchg_epoch(h) == 5
    finally:
        torch.cuda.synchronize()
        lib.qrc_xchg_destroy(h)


@pytest.mark.parametrize("peer_value", [9.25, 1.0])
def test_two_ranks_played_from_host(data, peer_value):
    """Rank 0 of two: its kernel writes its value into rank 1's slot array
    (a local buffer standing in for the peer) and takes rank 1's value from
    its own array, posted by the host beforehand."""
    import torch
    x, ctx = data
    lib = ctx.lib
    h = _xchg(lib, 0, 2)
    peer_slots = torch.zeros(4, dtype=torch.int64, device=x.device)      # 2 parities x 2 ranks
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        assert lib.qrc_xchg_debug_set_peer_ptr(h, 1, peer_slots.data_ptr()) == 0
        for _ in range(3):
            e = lib.qrc_xchg_epoch(h) + 1
            bits = int(np.array([peer_value], np.float32).view(np.uint32)[0])
            assert lib.qrc_xchg_debug_post(h, 1, e, bits) == 0
            assert lib.qrc_absmax_f32_allreduce(x.data_ptr(), x.numel(), out.data_ptr(), ctx.handle, h, None) == 0
            assert out.item() == max(5.5, peer_value)
            word = int(peer_slots[(e & 1) * 2 + 0].item()) & 0xFFFFFFFFFFFFFFFF
            assert word >> 32 == e and np.array([word & 0xFFFFFFFF], np.uint32).view(np.float32)[0] == 5.5
    finally:
        torch.cuda.synchronize()
        lib.qrc_xchg_destroy(h)


def test_missing_peer_times_out_with_nan(data):
    """No one posts rank 1's value: the wait gives up after about 2 s, the
    result is NaN, the error word is set, and the next plain call works."""
    import torch
    x, ctx = data
    lib = ctx.lib
    h = _xchg(lib, 0, 2)
    peer_slots = torch.zeros(4, dtype=torch.int64, device=x.device)
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        ctx.clear_diagnostics()
        assert lib.qrc_xchg_debug_set_peer_ptr(h, 1, peer_slots.data_ptr()) == 0
        assert lib.qrc_absmax_f32_allreduce(x.data_ptr(), x.numel(), out.data_ptr(), ctx.handle, h, None) == 0
        assert math.isnan(out.item())
        assert ctx.read_map(128)[H_XCHG_ERR] == 1
        assert ctx.absmax(x).item() == 5.5
        ctx.clear_diagnostics()
        assert ctx.read_map(128)[H_XCHG_ERR] == 0
    finally:
        torch.cuda.synchronize()
        lib.qrc_xchg_destroy(h)


def test_unmapped_peer_is_refused(data):
    import torch
    x, ctx = data
    lib = ctx.lib
    h = _xchg(lib, 1, 3)
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        assert lib.qrc_absmax_f32_allreduce(x.data_ptr(), x.numel(), out.data_ptr(), ctx.handle, h, None) == -5
    finally:
        lib.qrc_xchg_destroy(h)


def test_forty_ranks_played_from_host(data):
    """Rank 3 of 40: the last CTA's warp stores into every peer's slot array
    and polls its own 40 slots lane by lane (lanes 0..7 take two ranks each),
    so the maximum posted for any rank, including one polled on the second
    pass of a lane, reaches the result."""
    import torch
    x, ctx = data
    lib = ctx.lib
    world, rank = 40, 3
    h = _xchg(lib, rank, world)
    peers = torch.zeros((world, 2 * world), dtype=torch.int64, device=x.device)   # stand-ins for peer arrays
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        for p in range(world):
            if p != rank:
                assert lib.qrc_xchg_debug_set_peer_ptr(h, p, peers[p].data_ptr()) == 0
        for high in (37, 11, 3):                      # rank 37 is lane 5's second slot; 3 is this rank
            e = lib.qrc_xchg_epoch(h) + 1
            for p in range(world):
                if p != rank:
                    v = 6.0 + (4.0 if p == high else p / 64.0)
                    bits = int(np.array([v], np.float32).view(np.uint32)[0])
                    assert lib.qrc_xchg_debug_post(h, p, e, bits) == 0
            assert lib.qrc_absmax_f32_allreduce(x.data_ptr(), x.numel(), out.data_ptr(), ctx.handle, h, None) == 0
            want = 10.0 if high != rank else 6.0 + 39 / 64.0
            assert out.item() == np.float32(want), (high, out.item())
            torch.cuda.synchronize()
            par = e & 1                                # this rank's word went into every peer's array
            words = peers[:, par * world + rank].cpu().numpy().astype(np.uint64)
            for p in range(world):
                if p != rank:
                    assert int(words[p]) >> 32 == e and np.array([int(words[p]) & 0xFFFFFFFF], np.uint32).view(np.float32)[0] == 5.5
        assert int(ctx.read_map(128)[H_XCHG_ERR]) == 0
    finally:
        torch.cuda.synchronize()
        lib.qrc_xchg_destroy(h)
