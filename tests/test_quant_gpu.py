"""Fused amax -> FP8 e4m3 quantize: bytes, scale and amax bit-exact against
the CPU oracle; the device conversion against the OCP encoder exhaustively."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _f32_bits(t):
    import torch
    return int(t.detach().cpu().view(torch.int32).item()) & 0xFFFFFFFF


def _bf16_tensor(cuda, u16: np.ndarray):
    import torch
    return torch.from_numpy(u16.view(np.int16).copy()).to(cuda)


def _check(ctx, oracle, x_u16, cuda, offset_elems=0):
    import torch
    x = _bf16_tensor(cuda, x_u16)
    q, scale, amax = ctx.amax_quant_e4m3(x)
    qo, so = oracle.amax_quant_e4m3(x_u16)
    assert _f32_bits(amax) == int(np.array([oracle.absmax_bf16(x_u16)], np.float32).view(np.uint32)[0])
    assert _f32_bits(scale) == int(np.array([so], np.float32).view(np.uint32)[0])
    got = q.cpu().numpy()
    bad = np.nonzero(got != qo)[0]
    assert bad.size == 0, (bad[:8], got[bad[:8]], qo[bad[:8]], x_u16[bad[:8]])


@pytest.mark.parametrize("n", [0, 1, 2, 3, 7, 8, 9, 15, 16, 17, 4095, 4096, 8193, 1 << 20, (1 << 21) + 3])
def test_quant_sizes(cuda, qrc, oracle, n):
    x = oracle.normal_bf16(3, n, sigma=2.0)
    with qrc.SideAwareContext(device=0) as ctx:
        _check(ctx, oracle, x, cuda)


def test_quant_unaligned_views(cuda, qrc, oracle):
    import torch
    base = oracle.normal_bf16(4, (1 << 20) + 64, sigma=2.0)
    xb = _bf16_tensor(cuda, base)
    with qrc.SideAwareContext(device=0) as ctx:
        for off in (1, 3, 8, 13):
            view = xb[off:off + (1 << 20) - off]
            q = torch.empty(view.numel() + 16, dtype=torch.uint8, device=cuda)[off % 8:][:view.numel()]
            q2, scale, amax = ctx.amax_quant_e4m3(view, q=q)
            qo, so = oracle.amax_quant_e4m3(base[off:off + (1 << 20) - off])
            assert np.array_equal(q2.cpu().numpy(), qo)
            assert np.float32(scale.item()) == so


@pytest.mark.parametrize("vals", [
    [0x0000] * 33,                              # all zero -> scale 1, q 0
    [0x7FC0, 0x3F80, 0xFFC0] * 11,              # NaN ignored by amax, NaN -> 0x7F
    [0x7F80, 0x3F80, 0xBF80, 0xFF80] * 9,       # inf -> amax inf -> scale 1 -> +-448
    [0x8000, 0x0001, 0x8001] * 10,              # -0 and bf16 denormals
    [0x4380, 0xC3E0, 0x3C00] * 7,               # 256, -448, 2^-7
])
def test_quant_special_values(cuda, qrc, oracle, vals):
    x = np.array(vals, np.uint16)
    with qrc.SideAwareContext(device=0) as ctx:
        _check(ctx, oracle, x, cuda)


def test_quant_config4_full_shape(cuda, qrc, oracle):
    """bf16 [16384, 8192] normal(0,2) from seed 3: every byte and the scale."""
    import torch
    n = 16384 * 8192
    x = torch.empty(n, dtype=torch.int16, device=cuda)
    qrc.fill_normal_bf16(x, seed=3, sigma=2.0)
    host = x.cpu().numpy().view(np.uint16)
    with qrc.SideAwareContext(x) as ctx:
        q, scale, amax = ctx.amax_quant_e4m3(x)
        qo, so = oracle.amax_quant_e4m3(host)
        assert np.float32(scale.item()) == so
        assert np.array_equal(q.cpu().numpy(), qo)
        # same again (scratch reset between launches) in the ablation modes
        for mode in (1, 3, 0x20, 0x10, 0x30):
            ctx.mode = mode
            q2, s2, _ = ctx.amax_quant_e4m3(x)
            assert np.float32(s2.item()) == so and torch.equal(q, q2)
        ctx.mode = 0
        ctx.set_launch(1, 256)
        ctx.set_pipeline(6)              # amax pass through the bulk-copy ring
        q3, s3, _ = ctx.amax_quant_e4m3(x)
        assert np.float32(s3.item()) == so and torch.equal(q, q3)


@pytest.mark.slow
def test_e4m3_conversion_exhaustive(cuda, qrc, oracle):
    """All 2^32 float bit patterns through the device conversion equal the
    oracle's OCP encoder (RNE, satfinite, NaN -> 0x7F)."""
    import torch
    lib = qrc.load()
    chunk = 1 << 28
    out = torch.empty(chunk, dtype=torch.uint8, device=cuda)
    for c in range((1 << 32) // chunk):
        first = c * chunk
        bits = torch.arange(first, first + chunk, dtype=torch.int64, device=cuda).to(torch.int32)
        xs = bits.view(torch.float32)
        rc = lib.qrc_debug_cvt_e4m3(xs.data_ptr(), chunk, out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        got = out.cpu().numpy()
        want = oracle.e4m3_bits_range(first, chunk)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, [(hex(first + int(i)), hex(got[i]), hex(want[i])) for i in bad[:8]]
        del bits, xs


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_side_aware_quant_pass_on_mapped_buffer(cuda, qrc, oracle, mode):
    """The second pass reads side-aware when the input lies in the context's
    buffer: sizes and 16-byte-aligned offsets that give partial blocks, a
    head and a tail, against the oracle and the side-agnostic pass."""
    import torch
    total = (1 << 22) + 4096
    base = oracle.normal_bf16(6, total, sigma=2.0)
    xb = _bf16_tensor(cuda, base)
    with qrc.SideAwareContext(xb) as ctx:
        assert ctx.info["status"] == 0
        ctx.mode = mode
        for off, n in [(0, total), (8, total - 8), (4096, 1 << 22), (8, 8191), (0, 8), (24, (1 << 21) + 5)]:
            view = xb[off:off + n]
            q1, s1, a1 = ctx.amax_quant_e4m3(view)
            qo, so = oracle.amax_quant_e4m3(base[off:off + n])
            assert np.float32(s1.item()) == so
            assert np.array_equal(q1.cpu().numpy(), qo), (mode, off, n)
            assert ctx.lib.qrc_ctx_debug_quant_side_aware(ctx.handle, 0) == 0
            q2, s2, _ = ctx.amax_quant_e4m3(view)
            assert ctx.lib.qrc_ctx_debug_quant_side_aware(ctx.handle, 1) == 0
            assert torch.equal(q1, q2) and s1.item() == s2.item()
        # back-to-back launches: each pass leaves the queues reset
        for _ in range(3):
            q3, _, _ = ctx.amax_quant_e4m3(xb)
        assert np.array_equal(q3.cpu().numpy(), oracle.amax_quant_e4m3(base)[0])


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_fused_single_launch_quant(cuda, qrc, oracle, mode):
    """The single-launch fused kernel (amax, on-chip stash in tensor and
    shared memory, grid barrier, quantize): bit-exact against the oracle and
    the two-launch path on views with heads, tails and sizes below one 64 KiB
    block, and back to back while the maximum moves."""
    import torch
    total = (3 << 22) + 4096 + 40
    base = oracle.normal_bf16(9, total, sigma=2.0)
    xb = _bf16_tensor(cuda, base)
    with qrc.SideAwareContext(xb) as ctx:
        assert ctx.info["status"] == 0
        ctx.mode = mode
        for off, n in [(0, total), (8, total - 8), (32768, 1 << 22), (8, 8191), (0, 8), (24, (1 << 21) + 5),
                       (8, 40000), (0, 0)]:
            view = xb[off:off + n]
            q = torch.empty(n, dtype=torch.uint8, device=cuda)
            assert ctx.quant_launches(view, q) == 1
            q1, s1, a1 = ctx.amax_quant_e4m3(view, q=q)
            qo, so = oracle.amax_quant_e4m3(base[off:off + n])
            assert np.float32(s1.item()) == so, (mode, off, n)
            assert np.array_equal(q1.cpu().numpy(), qo), (mode, off, n)
            ctx.set_quant_fused(False)
            if n:
                assert ctx.quant_launches(view, q) == 2
            q2, s2, a2 = ctx.amax_quant_e4m3(view)
            ctx.set_quant_fused(True)
            assert torch.equal(q1, q2) and s1.item() == s2.item() and _f32_bits(a1) == _f32_bits(a2)
        for i in range(4):                           # back to back; the maximum moves every launch
            pos = [5, total // 2 + 3, total - 1, 70000][i]
            val = [0x4300, 0xC380, 0x4360, 0xC3C0][i]             # 128, -256, 224, -384
            saved = int(base[pos])
            base[pos] = val
            xb[pos] = int(np.array([val], np.uint16).view(np.int16)[0])
            q4, s4, a4 = ctx.amax_quant_e4m3(xb)
            qo, so = oracle.amax_quant_e4m3(base)
            assert np.float32(s4.item()) == so and np.array_equal(q4.cpu().numpy(), qo), i
            base[pos] = saved
            xb[pos] = int(np.array([saved], np.uint16).view(np.int16)[0])
        assert int(ctx.read_map(128)[99]) == 0      # no bounded wait gave up


def test_fused_quant_special_values_on_mapped_buffer(cuda, qrc, oracle):
    """NaN, infinities, -0 and denormals through the fused kernel."""
    import torch
    n = (1 << 21) + 48
    base = oracle.normal_bf16(10, n, sigma=2.0)
    xb = _bf16_tensor(cuda, base)
    with qrc.SideAwareContext(xb) as ctx:
        for vals in ([0x7FC0, 0xFFC0, 0x8000, 0x0001], [0x7F80, 0xFF80, 0x8001], [0x0000]):
            b = base.copy()
            idx = np.arange(0, n, 997)[: 64 * len(vals)]
            b[idx] = np.resize(np.array(vals, np.uint16), idx.size)
            if vals == [0x0000]:
                b[:] = 0
            xb.copy_(torch.from_numpy(b.view(np.int16)))
            assert ctx.quant_launches(xb) == 1
            q, s, a = ctx.amax_quant_e4m3(xb)
            qo, so = oracle.amax_quant_e4m3(b)
            assert _f32_bits(s) == int(np.array([so], np.float32).view(np.uint32)[0]), vals
            assert _f32_bits(a) == int(np.array([oracle.absmax_bf16(b)], np.float32).view(np.uint32)[0]), vals
            assert np.array_equal(q.cpu().numpy(), qo), vals
