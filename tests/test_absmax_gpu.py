"""Parity of the CUDA absmax path (through the C ABI) with the CPU oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MIB = 1 << 20
SIZES = [0, 1, 3, 4, 5, 1023, 4096, 8191, 8193, (1 << 19) - 1, (1 << 19) + 1,
         (2 * MIB) // 4 - 1, (2 * MIB) // 4, (2 * MIB) // 4 + 1, 3 * MIB + 7]
OFFSETS = [0, 1, 3, 1021]          # floats into the context's buffer
# read modes 0-3 with the schedule chosen by size (static shares at these
# sizes), and forced schedules: 0x10 static shares, 0x20 per-side queues,
# 0x30 static shares with a queued tail
MODES = [0, 1, 2, 3, 0x20, 0x21, 0x22, 0x10, 0x30, 0x31, 0x32]
# (blocks per SM, threads per block, bulk slots per warp; 0 = register loads)
SHAPES = [(1, 1024, 0), (2, 512, 0), (4, 256, 0), (1, 256, 6), (1, 512, 3), (1, 256, 2)]


def _bits(t):
    import torch
    return int(t.detach().cpu().view(torch.int32).item()) & 0xFFFFFFFF


@pytest.fixture(scope="module")
def buf(cuda, qrc):
    """64 MiB of uniform[-1,1) data with a side map."""
    import torch
    x = torch.empty(16 * MIB, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=11)
    torch.cuda.synchronize()
    ctx = qrc.SideAwareContext(x)
    yield x, ctx
    ctx.close()


def test_device_generators_match_oracle(cuda, qrc, oracle):
    import torch
    n = 1_000_003
    for seed, off in [(0, 0), (1, 7), (4, 3_000_000_000)]:
        x = torch.empty(n, dtype=torch.float32, device=cuda)
        qrc.fill_uniform(x, seed, offset=off)
        assert np.array_equal(x.cpu().numpy().view(np.uint32), oracle.uniform(seed, n, off).view(np.uint32))
        qrc.fill_normal(x, seed, sigma=2.0, offset=off)
        assert np.array_equal(x.cpu().numpy().view(np.uint32), oracle.normal(seed, n, 2.0, off).view(np.uint32))
        b = torch.empty(n, dtype=torch.int16, device=cuda)
        qrc.fill_normal_bf16(b, seed, sigma=2.0, offset=off)
        assert np.array_equal(b.cpu().numpy().view(np.uint16), oracle.normal_bf16(seed, n, 2.0, off))


def test_discovery_finds_two_sides(buf):
    x, ctx = buf
    info = ctx.info
    assert info["status"] == 0, info
    assert info["sms_side0"] > 0 and info["sms_side1"] > 0
    assert info["mask"] != 0 and info["mask"] & (info["chunk_bytes"]) and info["mask"] & (info["chunk_bytes"] - 1) == 0
    assert info["verify_mismatches"] * 8 <= info["verify_probes"]


def test_discovery_leaves_buffer_unchanged(cuda, qrc):
    import torch
    x = torch.empty(8 * MIB, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=3)
    before = x.clone()
    with qrc.SideAwareContext(x):
        torch.cuda.synchronize()
    assert torch.equal(before.view(torch.int32), x.view(torch.int32))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", SHAPES)
def test_absmax_parity_sizes_offsets(buf, oracle, mode, shape):
    import torch
    x, ctx = buf
    ctx.mode = mode
    ctx.set_pipeline(0)
    ctx.set_launch(shape[0], shape[1])
    ctx.set_pipeline(shape[2])
    host = x.cpu().numpy()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    for off in OFFSETS:
        for n in SIZES:
            ctx.absmax(x[off:off + n] if n else x[off:off], out=out, n=n)
            got = _bits(out)
            want = oracle.absmax_bits(host[off:off + n])
            assert got == want, (mode, shape, off, n, hex(got), hex(want))
    ctx.mode = 0
    ctx.set_pipeline(0)
    ctx.set_launch(1, 1024)


def test_pipeline_argument_checks(buf):
    x, ctx = buf
    import quickruncuda_b200 as q
    with pytest.raises(q.QrcError):
        ctx.set_pipeline(1)              # a ring needs at least two slots
    with pytest.raises(q.QrcError):
        ctx.set_pipeline(6)              # 1024 threads x 6 slots exceeds shared memory
    ctx.set_launch(1, 256)
    ctx.set_pipeline(6)
    with pytest.raises(q.QrcError):
        ctx.set_launch(2, 256)           # two CTAs per SM cannot both hold the ring
    ctx.set_pipeline(0)
    ctx.set_launch(1, 1024)


def test_bulk_pipeline_full_buffer_and_outliers(buf, oracle):
    import torch
    x, ctx = buf
    ctx.set_launch(1, 256)
    ctx.set_pipeline(6)
    saved = x[-1].clone()
    try:
        for mode in MODES:
            ctx.mode = mode
            for p in (0, 4095, 4096, x.numel() - 1):
                old = x[p].clone()
                x[p] = 1e30
                assert ctx.absmax(x).item() == np.float32(1e30), (mode, p)
                x[p] = old
        m = ctx.read_map(128)
        assert m[99] == 0                # no bounded wait gave up
    finally:
        x[-1] = saved
        ctx.mode = 0
        ctx.set_pipeline(0)
        ctx.set_launch(1, 1024)


def test_absmax_outlier_positions(buf, oracle):
    """An outlier planted at the first, last or any element is found: every
    element is read."""
    import torch
    x, ctx = buf
    n = 3 * MIB + 5
    view = x[2:2 + n]
    saved = view.clone()
    rng = np.random.default_rng(1)
    positions = [0, 1, n - 1, n - 2, 1024, 2047, 2048] + rng.integers(0, n, 40).tolist()
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    try:
        for mode in MODES:
            ctx.mode = mode
            for p in positions:
                view[p] = -9.0 - (p % 7)
                ctx.absmax(view, out=out)
                assert out.item() == 9.0 + (p % 7), (mode, p)
                view[p] = saved[p]
    finally:
        view.copy_(saved)
        ctx.mode = 0


@pytest.mark.parametrize("vals,expect_bits", [
    ([float("nan")] * 7, 0),
    ([-0.0] * 9, 0),
    ([0.5, float("inf"), float("nan")], 0x7F800000),
    ([1.401298464324817e-45, -2.802596928649634e-45, 0.0], 2),   # denormals kept: bits 1, 2
    ([float("nan"), -3.0, 2.0], 0x40400000),
])
def test_absmax_special_values(cuda, qrc, oracle, vals, expect_bits):
    import torch
    base = torch.zeros(1 << 16, dtype=torch.float32, device=cuda)
    v = torch.tensor(vals, dtype=torch.float32)
    with qrc.SideAwareContext(device=0) as ctx:
        for pos in (0, 4097, (1 << 16) - len(vals)):
            base.zero_()
            base[pos:pos + len(vals)] = v.to(cuda)
            for mode in MODES:
                ctx.mode = mode
                out = ctx.absmax(base)
                assert _bits(out) == expect_bits == oracle.absmax_bits(base.cpu().numpy())


def test_absmax_signalling_nan_and_random_bits(cuda, qrc, oracle):
    import torch
    rng = np.random.default_rng(9)
    u = rng.integers(0, 2 ** 32, size=(1 << 22) + 3, dtype=np.uint64).astype(np.uint32)
    u[::1000] = 0x7F800001          # signalling NaNs
    x = torch.from_numpy(u.view(np.float32)).to(cuda)
    with qrc.SideAwareContext(x) as ctx:
        for mode in MODES:
            ctx.mode = mode
            assert _bits(ctx.absmax(x)) == oracle.absmax_bits(u.view(np.float32))


@pytest.mark.parametrize("overlap", [1, 0])
def test_back_to_back_launches_reset_scratch(buf, oracle, overlap):
    """Each launch leaves queues, ticket and accumulator at zero, so results
    of consecutive launches on different data are independent (the reference
    relied on stale scratch, tests/side_aware.cu:371-374).  With programmatic
    dependent launch (overlap=1) each launch still sees the previous one's
    reset and the tensor writes between launches."""
    import torch
    x, ctx = buf
    ctx.set_overlap(overlap)
    n = 4 * MIB
    view = x[:n]
    saved = view.clone()
    outs = torch.empty(64, dtype=torch.float32, device=x.device)
    try:
        for i in range(64):
            view[(i * 7919) % n] = float(100 - i)     # decreasing maxima
            ctx.absmax(view, out=outs[i:i + 1])
            view[(i * 7919) % n] = saved[(i * 7919) % n]
        assert outs.cpu().tolist() == [float(100 - i) for i in range(64)]
    finally:
        view.copy_(saved)
        ctx.set_overlap(1)


def test_context_without_map_and_foreign_range(cuda, qrc, oracle):
    import torch
    x = torch.empty(5 * MIB + 3, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=21)
    x[12345] = -42.0
    want = oracle.absmax_bits(x.cpu().numpy())
    with qrc.SideAwareContext(device=0) as ctx:        # no buffer: side-agnostic
        assert ctx.info["status"] == 100
        assert _bits(ctx.absmax(x)) == want
    y = torch.empty(4 * MIB, dtype=torch.float32, device=cuda)
    with qrc.SideAwareContext(y) as ctx:              # map of another buffer
        assert _bits(ctx.absmax(x)) == want


def test_host_buffer_entry_point(cuda, qrc, oracle):
    import torch
    x = oracle.uniform_with_outlier(5, 9 * MIB + 1, 7.5)
    with qrc.SideAwareContext(device=0) as ctx:
        assert ctx.absmax_host(x) == 7.5
        pinned = torch.from_numpy(x).pin_memory()
        assert ctx.absmax_host(pinned) == 7.5
        assert ctx.absmax_host(x[:1000]) == oracle.absmax(x[:1000])
        assert ctx.absmax_host(x[:0]) == 0.0


def test_host_buffer_chunks_and_boundaries(cuda, qrc, oracle):
    """The host path copies 256 MiB chunks (64 Mi floats) and reduces each as
    it lands: the maximum must survive at every chunk edge, in a ragged last
    chunk, and after the staging was reserved larger than the input."""
    import torch
    from quickruncuda_b200 import _native as nat
    chunk = 64 * MIB
    n = 4 * chunk + 12345
    x = torch.from_numpy(oracle.uniform(6, n)).pin_memory()
    with qrc.SideAwareContext(device=0) as ctx:
        nat.check(ctx.lib, "qrc_host_reserve", ctx.lib.qrc_host_reserve(ctx.handle, n + chunk))
        for pos in (0, chunk - 1, chunk, 3 * chunk + 7, n - 1):
            x[pos] = -9.25
            got = ctx.absmax_host(x)
            assert np.float32(got) == oracle.absmax(x.numpy()) == np.float32(9.25), pos
            x[pos] = 0.5
        assert np.float32(ctx.absmax_host(x)) == oracle.absmax(x.numpy())
        assert np.float32(ctx.absmax_host(x[:chunk + 3])) == oracle.absmax(x[:chunk + 3].numpy())


def test_read_stream_reads_every_word(cuda, qrc, oracle):
    """The read-ceiling kernel of the bench: every shape XORs every 32-bit
    word of the buffer exactly once."""
    import torch
    from quickruncuda_b200 import _native as nat
    lib = nat.load()
    n = 8 * MIB + 4 * 37
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=12)
    want = int(np.bitwise_xor.reduce(x.cpu().numpy().view(np.uint32)))
    sink = torch.zeros(1, dtype=torch.int32, device=cuda)
    for depth, threads, bps in ((8, 1024, 1), (4, 1024, 2), (16, 512, 1), (32, 256, 1)):
        sink.zero_()
        assert lib.qrc_debug_read_stream(x.data_ptr(), 4 * n, depth, threads, bps, sink.data_ptr(), None) == 0
        torch.cuda.synchronize()
        assert int(sink.item()) & 0xFFFFFFFF == want, (depth, threads, bps)
    assert lib.qrc_debug_read_stream(x.data_ptr(), 4 * n, 8, 512, 1, sink.data_ptr(), None) == -1


def _cov_expect(addr: int, nbytes: int, unit: int = 2):
    a = np.arange(addr, addr + nbytes, unit, dtype=np.uint64)
    with np.errstate(over="ignore"):
        a ^= a >> np.uint64(31); a *= np.uint64(0x7FB5D329728EA185)
        a ^= a >> np.uint64(27); a *= np.uint64(0x81DADEF4BC2DD44D)
        a ^= a >> np.uint64(33)
    return int(np.bitwise_xor.reduce(a)) if a.size else 0


@pytest.mark.parametrize("mode", MODES)
def test_checked_build_every_byte_once_in_bounds(cuda, qrc, oracle, mode):
    """Checked build: no access leaves [A, A+4n), the bytes read sum to 4n and
    the XOR of per-address hashes equals that of the input range, so every
    2-byte unit is read an odd number of times and the byte count rules out
    repeats."""
    import torch
    x = torch.empty(6 * MIB, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=5)
    host = x.cpu().numpy()
    H_ERR, H_COV_BYTES, H_COV_XOR = 96, 100, 102
    with qrc.SideAwareContext(x, checked=True) as ctx:
        assert ctx.lib.qrc_is_checked_build() == 1
        ctx.mode = mode
        for off, n in [(0, 6 * MIB), (1, 6 * MIB - 1), (3, 2 * MIB + 5), (517, 8193), (0, 3), (7, 0)]:
            ctx.clear_diagnostics()
            view = x[off:off + n]
            out = ctx.absmax(view, n=n)
            m = ctx.read_map(128)
            assert m[H_ERR] == 0, (off, n)
            cov_bytes = int(m[H_COV_BYTES]) | (int(m[H_COV_BYTES + 1]) << 32)
            cov_xor = int(m[H_COV_XOR]) | (int(m[H_COV_XOR + 1]) << 32)
            assert cov_bytes == 4 * n
            assert cov_xor == _cov_expect(view.data_ptr(), 4 * n)
            assert _bits(out) == oracle.absmax_bits(host[off:off + n])


@pytest.mark.slow
def test_full_size_config2(cuda, qrc, oracle):
    """1e9 floats uniform[-1,1) seed 1 with the seeded outlier: exact result,
    all modes, against the oracle on the host copy."""
    import torch
    n = 1_000_000_000
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=1)
    i, s = qrc.outlier(1, n)
    x[i] = 7.5 * s
    want = oracle.absmax_bits(x.cpu().numpy())
    assert want == 0x40F00000
    with qrc.SideAwareContext(x) as ctx:
        assert ctx.info["status"] == 0, ctx.info
        for mode in MODES:
            ctx.mode = mode
            assert _bits(ctx.absmax(x)) == want
    del x
    torch.cuda.empty_cache()


def test_beyond_2_pow_32_elements(cuda, qrc):
    """17 GB: element indices past 2^32 (64-bit address arithmetic in the
    walks and the tail), every schedule; the planted outlier is the answer."""
    import torch
    n = (1 << 32) + 3
    x = torch.empty(n, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=17)
    try:
        with qrc.SideAwareContext(x) as ctx:
            for pos, val in [((1 << 32) + 1, -9.5), (n - 1, 11.25), (123, 3.0)]:
                old = float(x[pos].item())
                x[pos] = val
                for mode in (0, 0x10, 0x20, 0x30, 3):
                    ctx.mode = mode
                    assert ctx.absmax(x).item() == abs(val), (mode, pos)
                x[pos] = old
    finally:
        del x
        torch.cuda.empty_cache()
