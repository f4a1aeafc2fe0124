"""PyTorch custom operators over the C ABI: `torch.ops.qrc.absmax`,
`torch.ops.qrc.reduce` and `torch.ops.qrc.amax_quant_e4m3`.

These are for callers that hold tensors rather than raw buffers, such as a
quantized-inference stack computing per-tensor FP8 scales.  They are opaque
to torch.compile: the fake implementations give output shapes and dtypes, and
the CUDA implementations call libqrc_b200.so on the tensor's current stream.
There is no CPU implementation, so a CPU tensor is an error.

Side discovery runs once per allocation.  The operators keep a small cache of
contexts keyed by (device, storage base, storage size).  A tensor whose
storage was freed and whose addresses came back in a new allocation reuses
the old map; results stay exact, because the map decides only which die reads
which bytes.  `clear_context_cache()` drops the cache.  As with one context,
two calls on the same storage that run at the same time on different streams
share its scratch and race; calls on one stream are ordered.
"""
from __future__ import annotations

import collections
import threading

import torch

from .api import SideAwareContext

_CACHE_PER_DEVICE = 16
_cache: "collections.OrderedDict[tuple, SideAwareContext]" = collections.OrderedDict()
_lock = threading.Lock()


def _context_for(x: torch.Tensor) -> SideAwareContext:
    """The cached context of x's storage (created, with discovery, on first use)."""
    st = x.untyped_storage()
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    key = (dev, int(st.data_ptr()), int(st.nbytes()))
    with _lock:
        ctx = _cache.get(key)
        if ctx is not None:
            _cache.move_to_end(key)
            return ctx
        with torch.cuda.device(dev):
            # an empty storage gets a context without a map (side-agnostic)
            ctx = SideAwareContext(key[1] or None, device=dev, nbytes=key[2] or None,
                                   stream=torch.cuda.current_stream(dev))
        _cache[key] = ctx
        mine = [k for k in _cache if k[0] == dev]
        while len(mine) > _CACHE_PER_DEVICE:
            _cache.pop(mine.pop(0)).close()
        return ctx


def clear_context_cache() -> None:
    with _lock:
        while _cache:
            _cache.popitem()[1].close()


def _check_cuda(x: torch.Tensor, dtypes, name: str) -> None:
    if x.device.type != "cuda":
        raise RuntimeError(f"qrc::{name} needs a CUDA tensor, got {x.device}")
    if x.dtype not in dtypes:
        raise RuntimeError(f"qrc::{name} needs dtype in {dtypes}, got {x.dtype}")
    if not x.is_contiguous():
        raise RuntimeError(f"qrc::{name} needs a contiguous tensor")


@torch.library.custom_op("qrc::absmax", mutates_args=(), device_types="cuda")
def absmax(x: torch.Tensor) -> torch.Tensor:
    """max |x| over all elements of a float32 CUDA tensor, as a 0-dim float32
    tensor (NaN elements are ignored; an empty tensor gives 0)."""
    _check_cuda(x, (torch.float32,), "absmax")
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    ctx = _context_for(x)
    ctx.absmax(x, out=out, stream=torch.cuda.current_stream(x.device))
    return out.view(())


@absmax.register_fake
def _(x: torch.Tensor) -> torch.Tensor:
    return x.new_empty((), dtype=torch.float32)


_REDUCE_DTYPES = {"absmax": torch.float32, "max": torch.float32, "min": torch.float32,
                  "sum": torch.float64, "sumsq": torch.float64}


@torch.library.custom_op("qrc::reduce", mutates_args=(), device_types="cuda")
def reduce(x: torch.Tensor, op: str) -> torch.Tensor:
    """Side-aware reduction of a float32 CUDA tensor: op 'absmax', 'max',
    'min' (0-dim float32, NaN elements skipped) or 'sum', 'sumsq' (0-dim
    float64, accumulated in double)."""
    _check_cuda(x, (torch.float32,), "reduce")
    if op not in _REDUCE_DTYPES:
        raise RuntimeError(f"qrc::reduce: unknown op {op!r}")
    ctx = _context_for(x)
    out = ctx.reduce(x, op, stream=torch.cuda.current_stream(x.device))
    return out.view(())


@reduce.register_fake
def _(x: torch.Tensor, op: str) -> torch.Tensor:
    if op not in _REDUCE_DTYPES:
        raise RuntimeError(f"qrc::reduce: unknown op {op!r}")
    return x.new_empty((), dtype=_REDUCE_DTYPES[op])


@torch.library.custom_op("qrc::amax_quant_e4m3", mutates_args=(), device_types="cuda")
def amax_quant_e4m3(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-tensor FP8 quantize of a bf16 CUDA tensor: returns (q, scale,
    amax) with q = e4m3(x * scale) (round to nearest even, saturating) in
    x's shape, scale = 448 / amax (1 when amax is 0 or infinite) and amax =
    max |x|, both 0-dim float32."""
    _check_cuda(x, (torch.bfloat16,), "amax_quant_e4m3")
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    ctx = _context_for(x)
    ctx.amax_quant_e4m3(x, q=q, scale=scale, amax=amax, stream=torch.cuda.current_stream(x.device))
    return q.view(torch.float8_e4m3fn), scale.view(()), amax.view(())


@amax_quant_e4m3.register_fake
def _(x: torch.Tensor):
    return (x.new_empty(x.shape, dtype=torch.float8_e4m3fn), x.new_empty((), dtype=torch.float32),
            x.new_empty((), dtype=torch.float32))
