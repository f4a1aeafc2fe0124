"""The PyTorch custom operators on the GPU: torch.ops.qrc.absmax against the
oracle (bit-exact), torch.ops.qrc.amax_quant_e4m3 against the context call and
the oracle, and both inside torch.compile."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(t):
    import torch
    return int(t.detach().cpu().reshape(1).view(torch.int32).item()) & 0xFFFFFFFF


def test_absmax_op_matches_oracle(cuda, qrc, oracle):
    import torch
    import quickruncuda_b200.torch_ops as ops
    x = torch.empty(3 * (1 << 20) + 5, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=8)
    x[12345] = -6.25
    host = x.cpu().numpy()
    assert _bits(torch.ops.qrc.absmax(x)) == oracle.absmax_bits(host)
    # views: an offset slice and a 2-D reshape of the same storage
    v = x[1000:1000 + 777777]
    assert _bits(torch.ops.qrc.absmax(v)) == oracle.absmax_bits(host[1000:1000 + 777777])
    m = x[:3 * (1 << 20)].view(3, 1 << 20)
    assert _bits(torch.ops.qrc.absmax(m)) == oracle.absmax_bits(host[:3 << 20])
    assert _bits(torch.ops.qrc.absmax(x[:0])) == 0
    # two calls in a row on the same storage reuse one context
    before = len(ops._cache)
    torch.ops.qrc.absmax(x)
    assert len(ops._cache) == before
    ops.clear_context_cache()


def test_quant_op_matches_context_and_oracle(cuda, qrc, oracle):
    import torch
    import quickruncuda_b200.torch_ops as ops
    n = 1 << 22
    raw = torch.empty(n, dtype=torch.int16, device=cuda)
    qrc.fill_normal_bf16(raw, seed=3, sigma=2.0)
    x = raw.view(torch.bfloat16).view(1024, n // 1024)
    q, scale, amax = torch.ops.qrc.amax_quant_e4m3(x)
    assert q.shape == x.shape and q.dtype == torch.float8_e4m3fn
    qo, so = oracle.amax_quant_e4m3(raw.cpu().numpy().view(np.uint16))
    assert np.float32(scale.item()) == so
    assert np.array_equal(q.view(torch.uint8).reshape(-1).cpu().numpy(), qo)
    with qrc.SideAwareContext(raw) as ctx:
        q2, s2, a2 = ctx.amax_quant_e4m3(raw)
        assert torch.equal(q.view(torch.uint8).reshape(-1), q2) and s2.item() == scale.item()
        assert a2.item() == amax.item()
    ops.clear_context_cache()


def test_ops_inside_torch_compile(cuda, qrc, oracle):
    import torch
    import quickruncuda_b200.torch_ops as ops

    def f(x, xb):
        a = torch.ops.qrc.absmax(x * 2.0)
        q, s, _ = torch.ops.qrc.amax_quant_e4m3(xb)
        return a, q, s

    x = torch.empty(1 << 20, dtype=torch.float32, device=cuda)
    qrc.fill_uniform(x, seed=2)
    xb = x.to(torch.bfloat16)
    cf = torch.compile(f, backend="aot_eager", fullgraph=True)
    a, q, s = cf(x, xb)
    a0, q0, s0 = f(x, xb)
    assert _bits(a) == _bits(a0) == oracle.absmax_bits((x * 2.0).cpu().numpy())
    assert torch.equal(q.view(torch.uint8), q0.view(torch.uint8)) and s.item() == s0.item()
    ops.clear_context_cache()


def test_reduce_op_matches_oracle(cuda, qrc, oracle):
    import torch
    import quickruncuda_b200.torch_ops as ops
    x = torch.empty((1 << 21) + 9, dtype=torch.float32, device=cuda)
    qrc.fill_normal(x, seed=4, sigma=2.0)
    host = x.cpu().numpy()
    for op in ("max", "min"):
        got = torch.ops.qrc.reduce(x, op)
        assert got.dtype == torch.float32 and np.float32(got.item()) == oracle.reduce(op, host)
    for op in ("sum", "sumsq"):
        got = torch.ops.qrc.reduce(x, op)
        want, abs_sum = oracle.reduce(op, host)
        assert got.dtype == torch.float64
        assert abs(got.item() - want) <= host.size * 2.0 ** -52 * abs_sum
    ops.clear_context_cache()
