"""Sharded absmax over several GPUs: one process per GPU, each reducing its own
shard with the side-aware kernel, then one single-float max all-reduce.

The reference has no multi-GPU path (QuickRunCUDA.cpp:286 fixes device 0);
this is new: N GPUs, each with its own 1e9-float shard, and one maximum.
The exchange is one float per rank.
Two ways carry it:
  * PeerMax: inside the reduction kernel.  The last CTA of each rank stores
    its partial in every rank's exchange slots over NVLink (CUDA IPC
    mappings) and waits, bounded, for everyone's (qrc_absmax_f32_allreduce);
  * combine_max / MaxAllReduce: an NCCL max all-reduce after the kernel
    (MaxAllReduce on its own non-blocking communicator with a deadline).
Max over non-negative, non-NaN floats is exact and order-independent, so both
are bit-identical to a single-device reduction of the whole stream.
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

from . import _native as nat


@dataclass(frozen=True)
class ShardLayout:
    world: int
    n_per_rank: int
    seed: int
    outlier_rank: int
    outlier_local_index: int
    outlier_sign: int

    def offset(self, rank: int) -> int:
        """First global element index of `rank`'s shard."""
        return rank * self.n_per_rank

    def holds_outlier(self, rank: int) -> bool:
        return rank == self.outlier_rank


def shard_layout(world: int, n_per_rank: int, seed: int, outlier_index_fn) -> ShardLayout:
    """Rank r holds global elements [r*n, (r+1)*n) of the seed's stream; the one
    global outlier sits at outlier_index(seed, world*n), on the rank that holds
    that element.  `outlier_index_fn(seed, total) -> (index, sign)`."""
    if world < 1 or n_per_rank < 1:
        raise ValueError("world and n_per_rank must be positive")
    gi, sign = outlier_index_fn(seed, world * n_per_rank)
    return ShardLayout(world, n_per_rank, seed, gi // n_per_rank, gi % n_per_rank, sign)


def combine_max(value_tensor, group=None) -> None:
    """In-place max all-reduce of a 1-element float tensor (NCCL on GPUs, gloo
    on CPU ranks)."""
    import torch.distributed as dist
    dist.all_reduce(value_tensor, op=dist.ReduceOp.MAX, group=group)


class PeerLost(RuntimeError):
    """A rank stopped taking part in the sharded reduction: it announced that
    it left, or a max all-reduce did not complete before the deadline."""


class MaxAllReduce:
    """Max all-reduce of one float per rank that fails fast instead of
    waiting out a process-group timeout.

    * On NCCL it runs on its own communicator, created non-blocking
      (ncclConfig_t.blocking = 0) with the deadline as its timeout, so it can
      be aborted while a collective is outstanding without touching the
      caller's process group.
    * `enqueue` first asks the process group's store whether any rank has
      announced that it left (`leave`), so the others find out on the host,
      before their next launch.
    * `wait_all` polls the outstanding collectives until the deadline
      (`timeout_s`, from the first poll); a collective still pending then is
      aborted (the communicator with it) and PeerLost is raised.
    Every rank must call enqueue the same number of times in the same order,
    as with any collective.  Collective construction.
    """

    _instances = 0          # same count on every rank: construction is collective

    def __init__(self, group=None, timeout_s: float = 10.0, own_communicator: bool = True):
        import torch.distributed as dist
        from datetime import timedelta
        MaxAllReduce._instances += 1
        self.left_key = f"qrc/sharded/left/{MaxAllReduce._instances}"
        self.timeout_s = float(timeout_s)
        self.group = group
        self.pending = []
        self.aborted = False
        try:
            self.store = dist.distributed_c10d._get_default_store()
        except Exception:
            self.store = None
        if own_communicator and dist.get_backend(group) == "nccl":
            import torch
            opts = torch._C._distributed_c10d.ProcessGroupNCCL.Options()
            opts.config.blocking = 0
            ranks = dist.get_process_group_ranks(group) if group is not None else None
            self.group = dist.new_group(ranks=ranks, backend="nccl", pg_options=opts,
                                        timeout=timedelta(seconds=self.timeout_s))

    def left_count(self) -> int:
        """Ranks that announced they left (one store round trip)."""
        return int(self.store.add(self.left_key, 0)) if self.store is not None else 0

    def check_peers(self) -> None:
        if self.aborted:
            raise PeerLost("the max all-reduce was aborted earlier")
        n = self.left_count()
        if n:
            raise PeerLost(f"{n} rank(s) left the sharded reduction")

    def enqueue(self, value_tensor) -> None:
        """Start the max all-reduce of `value_tensor` in place.  The current
        stream waits for it (later work sees the result); the host does not."""
        import torch.distributed as dist
        self.check_peers()
        work = dist.all_reduce(value_tensor, op=dist.ReduceOp.MAX, group=self.group, async_op=True)
        if value_tensor.is_cuda:
            work.wait()                 # stream order only (a CPU tensor's wait would block the host)
        self.pending.append(work)

    def wait_all(self) -> None:
        """Host wait for every enqueued collective, bounded by the deadline."""
        deadline = time.monotonic() + self.timeout_s
        for work in self.pending:
            while not work.is_completed():
                if time.monotonic() > deadline:
                    self.abort()
                    raise PeerLost(f"max all-reduce not complete after {self.timeout_s:.1f} s")
                time.sleep(1e-4)
            try:
                work.wait()             # completed: returns at once, or raises the collective's error
            except Exception as e:
                self.abort()
                raise PeerLost(f"max all-reduce failed: {e}") from e
        self.pending.clear()

    def leave(self) -> None:
        """Announce that this rank takes part in no further reductions (call
        between steps, with nothing of this rank's in flight)."""
        if self.store is not None:
            self.store.add(self.left_key, 1)

    def abort(self) -> None:
        """Abort this object's communicator (outstanding collectives end with
        an error); the caller's process group is not touched."""
        import torch.distributed as dist
        self.aborted = True
        self.pending.clear()
        if self.group is not None:
            try:
                dist.distributed_c10d._abort_process_group(self.group)
            except Exception:
                pass


def sharded_absmax(ctx, shard, out, group=None):
    """Side-aware absmax of this rank's shard into `out` (1-element CUDA
    float32 tensor), then the max over all ranks.  Every rank must call it in
    the same order."""
    ctx.absmax(shard, out=out)
    combine_max(out, group)
    return out


class PeerMax:
    """Cross-GPU maximum taken inside the reduction kernel (qrc_xchg).  Built
    collectively: every rank of `group` must construct it, call `absmax` the
    same number of times in the same order, and `close` it."""

    def __init__(self, ctx, group=None):
        import torch.distributed as dist
        self.ctx, self.lib, self.group = ctx, ctx.lib, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        h = ctypes.c_void_p()
        nat.check(self.lib, "qrc_xchg_create", self.lib.qrc_xchg_create(ctypes.byref(h), ctx.device, self.rank,
                                                                       self.world))
        self._h = h
        buf = ctypes.create_string_buffer(64)
        nat.check(self.lib, "qrc_xchg_get_handle", self.lib.qrc_xchg_get_handle(h, buf))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(buf.raw), group=group)
        for p in range(self.world):
            if p != self.rank:
                nat.check(self.lib, "qrc_xchg_set_peer", self.lib.qrc_xchg_set_peer(h, p, handles[p]))

    @classmethod
    def try_create(cls, ctx, group=None):
        """A PeerMax on every rank, or None on every rank when any rank could
        not map its peers (the caller then uses combine_max)."""
        import torch.distributed as dist
        px, ok = None, True
        try:
            px = cls(ctx, group)
        except Exception:
            ok = False
        oks = [None] * dist.get_world_size(group)
        dist.all_gather_object(oks, ok, group=group)
        if all(oks):
            return px
        if px is not None:
            px.close(barrier=False)
        return None

    def absmax(self, x, out, n=None, stream=None):
        """max |x| over every rank's x, into `out` on every rank.  NaN when a
        peer's value did not arrive within the bounded wait."""
        from .api import _ptr, _stream_handle
        n = int(x.numel()) if n is None else n
        nat.check(self.lib, "qrc_absmax_f32_allreduce",
                  self.lib.qrc_absmax_f32_allreduce(_ptr(x) or None, n, _ptr(out), self.ctx.handle, self._h,
                                                    _stream_handle(stream, self.ctx.device) or None))
        return out

    def close(self, barrier: bool = True) -> None:
        """Collective: waits until every rank is done before the slots go."""
        if getattr(self, "_h", None) is None:
            return
        import torch
        torch.cuda.synchronize(self.ctx.device)
        if barrier:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        self.lib.qrc_xchg_destroy(self._h)
        self._h = None
