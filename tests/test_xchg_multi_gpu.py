"""Multi-GPU paths, one process per GPU (skipped when the box has fewer GPUs):

* the in-kernel cross-GPU maximum at 2, 4 and 8 ranks: CUDA IPC mappings of
  each other's exchange slots, the result compared with an NCCL max
  all-reduce of the same per-GPU values while the maximum moves between
  ranks;
* the fail-fast NCCL combine (MaxAllReduce): a rank that leaves between steps
  is reported to the survivor on the host, before its next launch, within
  10 s.  NVLS is off in NCCL for these runs; no kernel or collective of the
  leaving rank is in flight when it goes."""
import os
import time

import pytest

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        import quickruncuda_b200 as qrc
        from quickruncuda_b200.sharded import PeerMax
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        n = (1 << 22) + 5 * rank
        x = torch.empty(n, dtype=torch.float32, device=dev)
        qrc.fill_uniform(x, seed=30 + rank)
        ctx = qrc.SideAwareContext(x)
        px = PeerMax(ctx)
        out = torch.empty(1, dtype=torch.float32, device=dev)
        ref = torch.empty(1, dtype=torch.float32, device=dev)
        ok = True
        for i in range(20):
            x[(i * 7919 + rank) % n] = float(10 + i * world + rank)     # the maximum moves between ranks
            px.absmax(x, out)
            ctx.absmax(x, out=ref)
            dist.all_reduce(ref, op=dist.ReduceOp.MAX)
            ok &= out.item() == ref.item() == float(10 + i * world + world - 1)
        px.close()
        ctx.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as e:                      # reported to the parent
        q.put((rank, repr(e)))
    finally:
        q.close()
        q.join_thread()


def _spawn(target, world, extra=()):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() * 7 + world) % 1000
    procs = [ctx.Process(target=target, args=(r, world, port, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_in_kernel_max_matches_nccl(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(_rank, world)
    assert res == {r: True for r in range(world)}, res


def _leaving_rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        import quickruncuda_b200 as qrc
        from quickruncuda_b200.sharded import MaxAllReduce, PeerLost
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        x = torch.empty(1 << 22, dtype=torch.float32, device=dev)
        qrc.fill_uniform(x, seed=40 + rank)
        x[rank] = 3.0 + rank
        ctx = qrc.SideAwareContext(x)
        mar = MaxAllReduce(timeout_s=10.0)
        out = torch.empty(1, dtype=torch.float32, device=dev)
        for _ in range(3):
            ctx.absmax(x, out=out)
            mar.enqueue(out)
            mar.wait_all()
            assert out.item() == 3.0 + world - 1
        torch.cuda.synchronize()
        if rank == world - 1:                   # leaves between steps, nothing in flight
            mar.leave()
            q.put((rank, "left"))
            return
        time.sleep(1.0)                         # the next step comes after the other rank left
        t0 = time.monotonic()
        try:
            ctx.absmax(x, out=out)
            mar.enqueue(out)
            mar.wait_all()
            q.put((rank, "no failure reported"))
        except PeerLost:
            q.put((rank, ("reported", time.monotonic() - t0)))
        torch.cuda.synchronize()
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        q.close()
        q.join_thread()
        os._exit(0)                             # no collective teardown with a rank gone


def test_rank_that_leaves_is_reported_within_10s():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _spawn(_leaving_rank, 2)
    assert res[1] == "left", res
    assert isinstance(res[0], tuple) and res[0][0] == "reported" and res[0][1] < 10.0, res
