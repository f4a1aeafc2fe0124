"""The other reduction operators (qrc_reduce_f32: max, min, sum, sum of
squares) against the oracle.  max and min are bit-exact.  Sums are in double
with a launch-dependent order, so they are checked against the oracle's
compensated sum within n * 2^-52 * sum |term|: a single element missed or
added twice is far outside that bound."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MIB = 1 << 20
SIZES = [0, 1, 5, 1023, 8193, (1 << 19) + 1, (2 * MIB) // 4 + 1, 3 * MIB + 7]
OFFSETS = [0, 3]
# mode | schedule: side-aware automatic, page bits ignored, stream, queues,
# balanced, static
MODES = [0, 1, 3, 0x20, 0x30, 0x10]
# (blocks per SM, threads, bulk slots): one CTA per SM, two CTAs of 1024 per
# SM (a second wave re-enters SMs whose share is taken), 512, bulk ring
SHAPES = [(1, 1024, 0), (2, 1024, 0), (2, 512, 0), (1, 256, 6)]
OPS = ["max", "min", "sum", "sumsq"]


def _check(oracle, op, got, host):
    if op in ("max", "min"):
        want = oracle.reduce(op, host)
        assert np.array([got], np.float32).view(np.uint32)[0] == np.array([want], np.float32).view(np.uint32)[0], \
            (op, got, want)
    else:
        want, abs_sum = oracle.reduce(op, host)
        tol = max(host.size, 1) * 2.0 ** -52 * abs_sum + 1e-300
        assert abs(got - want) <= tol, (op, host.size, got, want, tol)


@pytest.fixture(scope="module")
def buf(cuda, qrc):
    import torch
    x = torch.empty(4 * MIB, dtype=torch.float32, device=cuda)
    qrc.fill_normal(x, seed=6, sigma=3.0)
    torch.cuda.synchronize()
    ctx = qrc.SideAwareContext(x)
    yield x, ctx
    ctx.close()


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", SHAPES)
def test_reduce_parity(buf, oracle, op, mode, shape):
    x, ctx = buf
    ctx.mode = mode
    ctx.set_pipeline(0)
    ctx.set_launch(shape[0], shape[1])
    ctx.set_pipeline(shape[2])
    host = x.cpu().numpy()
    try:
        for off in OFFSETS:
            for n in SIZES:
                out = ctx.reduce(x[off:off + n], op, n=n)
                _check(oracle, op, float(out.item()), host[off:off + n])
    finally:
        ctx.mode = 0
        ctx.set_pipeline(0)
        ctx.set_launch(1, 1024)


@pytest.mark.parametrize("vals", [
    [0.0, -0.0], [-0.0, 0.0, -0.0], [float("nan"), 1.0, float("-inf")], [float("inf"), -2.0],
    [float("nan")], [-1e-45, 1e-45], [3.0, float("nan"), -7.0, float("inf"), float("-inf")],
    [2.0, 3.0], [-2.0, -5.0],          # one sign only: partial batches must not add zeros
])
def test_reduce_special_values(cuda, qrc, oracle, vals):
    import torch
    pattern = np.array(vals, np.float32)
    host = np.resize(pattern, 3 * MIB + 11)           # repeated, so every CTA sees them
    x = torch.from_numpy(host).to(cuda)
    with qrc.SideAwareContext(x) as ctx:
        for mode in (0, 0x30, 3):
            ctx.mode = mode
            for op in OPS:
                got = float(ctx.reduce(x, op).item())
                if op in ("max", "min"):
                    _check(oracle, op, got, host)
                else:
                    want, _ = oracle.reduce(op, host)
                    if np.isnan(want):
                        assert np.isnan(got), (op, vals)
                    elif np.isinf(want):
                        assert got == want, (op, vals)
                    else:
                        _check(oracle, op, got, host)


def test_sum_every_byte_once_checked_build(cuda, qrc, oracle):
    """Checked build: the sum path reads every byte exactly once, including
    two CTAs per SM contending for the same static share."""
    import torch
    H_ERR, H_COV_BYTES = 96, 100
    x = torch.empty(6 * MIB, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=9)
    host = x.cpu().numpy()
    with qrc.SideAwareContext(x, checked=True) as ctx:
        for blocks, mode in [(1, 0), (2, 0), (2, 0x30), (1, 0x20)]:
            ctx.set_launch(blocks, 1024)
            ctx.mode = mode
            for off, n in [(0, 6 * MIB), (5, 6 * MIB - 9), (1, 8193)]:
                ctx.clear_diagnostics()
                got = float(ctx.reduce(x[off:off + n], "sum", n=n).item())
                m = ctx.read_map(128)
                assert m[H_ERR] == 0
                assert (int(m[H_COV_BYTES]) | (int(m[H_COV_BYTES + 1]) << 32)) == 4 * n, (blocks, mode, off, n)
                _check(oracle, "sum", got, host[off:off + n])
        ctx.set_launch(1, 1024)


@pytest.mark.parametrize("op,name", [(1, "max"), (2, "min"), (3, "sum"), (4, "sumsq")])
def test_kernel_file_operator_under_our_harness(tmp_path, oracle, op, name):
    """The drop-in kernel file compiled with -H '#define QRC_PLUGIN_OP n':
    C[0] holds the result as a float (sums rounded once from double)."""
    import json
    import subprocess
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    harness = root / "quickruncuda_b200" / "bin" / "qrc_harness"
    kernel = root / "quickruncuda_b200" / "csrc" / "side_aware_b200.cu"
    n = (1 << 21) + 3
    r = subprocess.run([str(harness), "-i", "-p", "-t", "1024", "-A", str(n), "-0", str(n), "-C", "1", "-T", "3",
                        "-H", f"#define QRC_PLUGIN_OP {op}", "--fill-a", "uniform:0:7.5", "--json", str(kernel)],
                       cwd=tmp_path, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    bits = json.loads(r.stdout.strip().splitlines()[-1])["c0_bits"]
    c0 = np.array([bits], np.uint32).view(np.float32)[0]
    host = oracle.uniform_with_outlier(0, n, 7.5)
    if name in ("max", "min"):
        assert c0 == oracle.reduce(name, host)
    else:
        want, abs_sum = oracle.reduce(name, host)
        assert abs(float(c0) - want) <= abs(want) * 2.0 ** -24 + n * 2.0 ** -52 * abs_sum, (c0, want)
