"""Host logic of the sharded reduction with world-size-2 gloo ranks on CPU:
shard layout, outlier placement and the max combine, plus a rank that leaves
early making the other rank's collective fail within its timeout instead of
hanging."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from quickruncuda_b200.sharded import shard_layout


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _outlier_fn():
    import quickruncuda_b200 as q
    return q.outlier


def test_layout_single_global_outlier():
    import quickruncuda_b200 as q
    for world in (1, 2, 4, 8):
        lay = shard_layout(world, 1_000_000_000, 4, q.outlier)
        gi, sign = q.outlier(4, world * 1_000_000_000)
        assert lay.outlier_rank == gi // 1_000_000_000 < world
        assert lay.offset(lay.outlier_rank) + lay.outlier_local_index == gi
        assert sum(lay.holds_outlier(r) for r in range(world)) == 1
        assert lay.outlier_sign == sign


def _worker(rank, world, port, n, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import quickruncuda_b200 as q
        from tests._oracle import Oracle
        orc = Oracle.load()
        lay = shard_layout(world, n, 4, q.outlier)
        shard = np.empty(n, np.float32)
        q.host_fill_uniform(shard, lay.seed, lay.offset(rank))
        if lay.holds_outlier(rank):
            shard[lay.outlier_local_index] = 7.5 * lay.outlier_sign
        # the per-shard reduction runs on the GPU in production; the oracle
        # stands in here so the test covers only the host-side combine
        local = torch.tensor([float(orc.absmax(shard))], dtype=torch.float32)
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
        result_q.put((rank, float(local.item()), float(orc.absmax(shard))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_combine_to_the_global_answer(oracle):
    world, n = 2, 300_001
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [rq.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    whole = oracle.uniform(4, world * n)
    import quickruncuda_b200 as q
    gi, sign = q.outlier(4, world * n)
    whole[gi] = 7.5 * sign
    assert all(r[1] == 7.5 == float(oracle.absmax(whole)) for r in res)
    assert sorted(r[2] == 7.5 for r in res) == [False, True]


def _leaver(rank, world, port, result_q):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = torch.ones(1)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)          # one good step together
    if rank == 1:
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()
        os._exit(0)                                     # leaves between steps
    t0 = time.time()
    try:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        result_q.put((rank, "no error"))
    except Exception as e:                               # gloo reports the lost peer / timeout
        result_q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


def test_rank_leaving_between_steps_fails_the_next_collective():
    world = 2
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, world, port, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(rq.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 30.0


def _max_allreduce_worker(rank, world, port, scenario, result_q):
    """MaxAllReduce on gloo ranks: `leave` (rank 1 announces it left after one
    step) or `stall` (rank 1 stays alive but skips the second collective)."""
    from datetime import timedelta
    from quickruncuda_b200.sharded import MaxAllReduce, PeerLost
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    mar = MaxAllReduce(timeout_s=2.0)
    t = torch.tensor([float(rank + 1)])
    mar.enqueue(t)
    mar.wait_all()
    ok = t.item() == float(world)
    if rank == 1:
        if scenario == "leave":
            mar.leave()
        result_q.put((rank, ("stepped", ok)))
        if scenario == "stall":
            time.sleep(6.0)
        result_q.close()
        result_q.join_thread()
        os._exit(0)
    time.sleep(0.5 if scenario == "leave" else 0.0)
    t0 = time.monotonic()
    try:
        mar.enqueue(t)
        mar.wait_all()
        result_q.put((rank, ("no failure", ok)))
    except PeerLost as e:
        result_q.put((rank, ("lost", ok, time.monotonic() - t0, str(e))))
    result_q.close()
    result_q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("scenario", ["leave", "stall"])
def test_max_allreduce_reports_a_lost_rank_fast(scenario):
    """A rank that announces it left is reported before the next collective
    starts; a rank that never joins the collective is reported when the
    deadline (2 s here) passes, not after the process-group timeout (30 s)."""
    world = 2
    ctx = mp.get_context("spawn")
    rq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_max_allreduce_worker, args=(r, world, port, scenario, rq)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(rq.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
    assert res[1] == ("stepped", True), res
    kind, ok, took, msg = res[0]
    assert kind == "lost" and ok, res
    if scenario == "leave":
        assert took < 1.0 and "left" in msg, res
    else:
        assert 1.5 < took < 10.0 and "not complete" in msg, res
