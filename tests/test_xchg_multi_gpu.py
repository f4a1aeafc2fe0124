"""The in-kernel cross-GPU maximum on two GPUs: one process per GPU, CUDA IPC
mappings of each other's exchange slots, and the result compared with an NCCL
max all-reduce of the same per-GPU values.  Skipped with fewer than 2 GPUs."""
import os

import pytest

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
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


def test_two_gpu_in_kernel_max_matches_nccl():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}, res
