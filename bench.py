"""Benchmark of the side-aware FP32 absmax on B200 (one JSON line on stdout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1: the 1e9-float workload (4 GB, uniform[-1,1) from seed 1, one outlier of
magnitude 7.5 at a seeded index).  A step is one reduction of the whole
buffer: one kernel launch through the C ABI (qrc_absmax_f32).
N > 1 (one process per GPU under torchrun): every rank holds 1e9 floats of the
seed-4 uniform stream (rank r: elements [r*1e9, (r+1)*1e9)), one global
outlier on a seeded rank; a step is the per-shard reduction plus a
single-float max all-reduce over NCCL.  Weak scaling.

`value` is whole-job GB/s with inputs resident in HBM (the 4 GB input is 32x
the 126 MB L2, so no flush is needed between steps).  `e2e` is the same metric
through qrc_absmax_f32_host: every step copies the 4 GB shard from pinned host
memory and reads the 4-byte result back.  `--impl reference` times the CPU
restatement of the reference reduction (oracle/, OpenMP on all host cores),
since the reference has no CPU implementation of this path.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_PER_GPU = 1_000_000_000
BYTES_PER_GPU = 4 * N_PER_GPU
OUTLIER = 7.5
METRIC = "FP32 absmax GB/s at 1e9 floats (% of B200 HBM peak) at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
# The kernel's automatic schedule: static per-SM shares alone up to this many
# input bytes (32,768 pairs of 8 KiB), static shares with a queued tail above.
STATIC_MAX_BYTES = 32768 * 8192
L2_NOTE = "input 4 GB per GPU > 126 MB L2 (no flush needed)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", default="side_aware", choices=["side_aware", "ignore_page_bits", "wrong_side", "stream"])
    ap.add_argument("--sched", default="auto", choices=["auto", "static", "queue", "balanced"],
                    help="work schedule: by size, fixed per-SM shares, per-side queues, or shares plus a queued tail")
    ap.add_argument("--collective", default="fused", choices=["fused", "nccl"],
                    help="N>1: cross-GPU max inside the kernel over NVLink peer stores, or an NCCL all-reduce")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-ablation", action="store_true")
    ap.add_argument("--no-quant", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch reductions in plain stream order (no programmatic dependent launch)")
    ap.add_argument("--e2e-steps", type=int, default=0, help="0 = min(10, max(3, steps // 100))")
    ap.add_argument("--n-per-gpu", type=int, default=N_PER_GPU,
                    help="floats per GPU (default 1e9; smaller sizes are for profiling captures)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def host_threads() -> int:
    """All host cores this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its workers; the CPU baseline must not inherit that)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name: str):
    """dram bytes per launch recorded from an ncu capture (profiles/<name>.md,
    line `traffic_bytes_per_launch: N`), or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """NVML sampler (read-only) for the timed region: SM clock, power and
    clock-event reasons."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x10: "sync_boost", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.01):
        self.ok = False
        self.samples = []
        self.period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()
        self._th = None

    def _reasons(self):
        nv = self.nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self.h))

    def _loop(self):
        while not self._stop.is_set():
            try:
                clk = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                pw = self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((clk, pw, self._reasons()))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._th = threading.Thread(target=self._loop, daemon=True)
            self._th.start()
        return self

    def __exit__(self, *exc):
        if self._th:
            self._stop.set()
            self._th.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        clks = sorted(s[0] for s in self.samples)
        reasons = 0
        for s in self.samples:
            reasons |= s[2]
        return {"sm_mhz": clks[len(clks) // 2], "sm_max_mhz": self.max_mhz,
                "reasons": [v for k, v in self.REASONS.items() if reasons & k],
                "samples": len(self.samples),
                "power_w_median": round(sorted(s[1] for s in self.samples)[len(self.samples) // 2], 1)}


# ---------------------------------------------------------------------------
# Reference arm: the CPU restatement of the reduction, all host cores
# ---------------------------------------------------------------------------

def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    from tests._oracle import Oracle
    orc = Oracle.load()
    n = args.n_per_gpu
    nbytes = 4 * n
    x = orc.uniform_with_outlier(1, n, OUTLIER)
    used = ctypes.c_int()
    fptr = x.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    nthr = host_threads()
    for _ in range(max(args.warmup, 1)):
        orc.lib.oracle_absmax_f32(fptr, n, nthr, ctypes.byref(used))
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = orc.lib.oracle_absmax_f32(fptr, n, nthr, ctypes.byref(used))
        times.append(time.perf_counter() - t0)
    assert r == OUTLIER, r
    total = sum(times)
    value = nbytes * len(times) / total / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / len(times), 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "absmax of 1e9 f32 uniform[-1,1) seed 1 + outlier 7.5 (one GPU's shard)",
                   "n": n, "bytes": nbytes},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": int(used.value), "kind": "port",
                         "sample": f"full 1e9-float buffer, {args.steps} passes (OpenMP restatement of "
                                   "tests/side_aware.cu:216-219; the reference has no CPU path)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import quickruncuda_b200 as q
    from quickruncuda_b200 import _native as nat

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.current_stream(dev)

    # ---- input shard, resident in HBM ----
    n = args.n_per_gpu
    nbytes = 4 * n
    x = torch.empty(n, dtype=torch.float32, device=dev)
    if world == 1:
        seed, offset = 1, 0
        gi, sign = q.outlier(seed, n)
        workload = f"absmax of {n} f32 uniform[-1,1) seed 1 + one outlier 7.5 at a seeded index"
    else:
        seed, offset = 4, rank * n
        gi, sign = q.outlier(seed, world * n)
        workload = f"sharded absmax: {world} x {n} f32 uniform[-1,1) seed 4, one global outlier 7.5, max all-reduce"
    q.fill_uniform(x, seed, offset=offset)
    if offset <= gi < offset + n:
        x[gi - offset] = OUTLIER * sign
    torch.cuda.synchronize()

    t0 = time.perf_counter()
    ctx = q.SideAwareContext(x, device=local)
    init_ms = 1e3 * (time.perf_counter() - t0)
    info = ctx.info
    ctx.mode = args.mode
    ctx.schedule = args.sched
    ctx.set_overlap(not args.no_overlap)
    out = torch.zeros(1, dtype=torch.float32, device=dev)
    px = None
    if world > 1 and args.collective == "fused":
        from quickruncuda_b200.sharded import PeerMax
        px = PeerMax.try_create(ctx)            # None on every rank if peers cannot be mapped
    collective = ("in-kernel NVLink peer max" if px is not None else "nccl_max_allreduce") if world > 1 else None

    def step():
        if px is not None:
            px.absmax(x, out)
            return
        ctx.absmax(x, out=out)
        if world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.MAX)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    assert out.item() == OUTLIER, f"warm-up result {out.item()} != {OUTLIER}"

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(end)
    tmax = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    ms_total = float(tmax.item())
    ms_per_step = ms_total / args.steps
    assert out.item() == OUTLIER, f"timed result {out.item()} != {OUTLIER}"
    value = world * nbytes / (ms_per_step / 1e3) / 1e9

    # ---- ablations on this rank (same kernel, other read modes) ----
    # Each read mode under each work schedule: the per-side queues move both
    # sides through the buffer in step, so with page bits ignored whole 2 MiB
    # pages are read from the far die at once; static shares spread the sides
    # over the buffer.
    ablation = {}
    if not args.no_ablation and world == 1:
        abl_steps = max(3, min(args.steps, 200))
        for m in ("side_aware", "ignore_page_bits", "wrong_side", "stream"):
            for sched in (("auto",) if m == "stream" else ("static", "balanced", "queue")):
                ctx.mode = m
                ctx.schedule = sched
                for _ in range(3):
                    ctx.absmax(x, out=out)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(stream)
                for _ in range(abl_steps):
                    ctx.absmax(x, out=out)
                e.record(stream)
                torch.cuda.synchronize()
                assert out.item() == OUTLIER
                gbs = round(nbytes / (s.elapsed_time(e) / abl_steps / 1e3) / 1e9, 2)
                if m == "stream":
                    ablation[m] = gbs
                else:
                    ablation.setdefault(m, {})[sched] = gbs
        ctx.mode = args.mode
        ctx.schedule = args.sched

    # ---- fused amax -> e4m3 quantize, bf16 [16384, 8192] normal(0, 2) seed 3 ----
    quant = None
    if not args.no_quant and world == 1:
        nq = 16384 * 8192
        xq = torch.empty(nq, dtype=torch.int16, device=dev)
        q.fill_normal_bf16(xq, seed=3, sigma=2.0)
        qout = torch.empty(nq, dtype=torch.uint8, device=dev)
        qscale = torch.empty(1, dtype=torch.float32, device=dev)
        qamax = torch.empty(1, dtype=torch.float32, device=dev)
        with q.SideAwareContext(xq, device=local) as cq:
            for _ in range(3):
                cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax)
            qsteps = max(3, min(args.steps, 300))
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            for _ in range(qsteps):
                cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax)
            e.record(stream)
            torch.cuda.synchronize()
        qms = s.elapsed_time(e) / qsteps
        qbytes = 2 * 2 * nq + nq          # two reads of the bf16 input (amax, then quantize) + one e4m3 write
        qgbs = qbytes / (qms / 1e3) / 1e9
        peak, _ = measured_peak()
        quant = {"workload": "bf16 [16384, 8192] normal(0,2) seed 3 -> e4m3 + scale", "ms": round(qms, 5),
                 "gbs": round(qgbs, 2), "algorithmic_bytes": qbytes, "launches_per_step": 2,
                 "roofline_frac": round(qgbs / peak, 4), "scale": float(qscale.item()), "amax": float(qamax.item())}
        del xq, qout

    # ---- end to end through the host-buffer C-ABI call ----
    e2e = None
    h_ptr = None
    if not args.no_e2e:
        e2e_steps = args.e2e_steps or min(10, max(3, args.steps // 100))
        host = torch.empty(n, dtype=torch.float32, pin_memory=True)
        q.host_fill_uniform(host, seed, offset)
        if offset <= gi < offset + n:
            host[gi - offset] = OUTLIER * sign
        res = ctypes.c_float()
        lib = ctx.lib

        def e2e_step():
            rc = lib.qrc_absmax_f32_host(ctypes.c_void_p(host.data_ptr()), n, ctypes.byref(res), ctx.handle,
                                         ctypes.c_void_p(stream.cuda_stream))
            nat.check(lib, "qrc_absmax_f32_host", rc)
            if world > 1:
                t = torch.tensor([res.value], dtype=torch.float32, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                return float(t.item())
            return res.value

        r0 = e2e_step()                     # first call allocates and maps the staging buffer
        assert r0 == OUTLIER, r0
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(e2e_steps):
            r0 = e2e_step()
        e.record(stream)
        torch.cuda.synchronize()
        assert r0 == OUTLIER
        t = torch.tensor([s.elapsed_time(e)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item()) / e2e_steps
        e2e = {"value": round(world * nbytes / (e2e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": world * nbytes, "d2h_bytes_per_step": world * 4,
               "steps": e2e_steps, "ms_per_step": round(e2e_ms, 3),
               "path": "qrc_absmax_f32_host (pinned host -> device staging -> side-aware kernel -> host)"}
        h_ptr = host

    # ---- CPU baseline on the same host data (rank 0, N = 1 only) ----
    cpu = None
    if world == 1 and not args.no_cpu:
        from tests._oracle import Oracle
        orc = Oracle.load()
        if h_ptr is None:
            h_ptr = torch.empty(n, dtype=torch.float32)
            q.host_fill_uniform(h_ptr, seed, offset)
            h_ptr[gi] = OUTLIER * sign
        fptr = ctypes.cast(ctypes.c_void_p(h_ptr.data_ptr()), ctypes.POINTER(ctypes.c_float))
        used = ctypes.c_int()
        nthr = host_threads()
        t0 = time.perf_counter()
        r = orc.lib.oracle_absmax_f32(fptr, n, nthr, ctypes.byref(used))
        t1 = time.perf_counter() - t0
        reps = int(min(10, max(3, 10.0 // max(t1, 1e-3))))
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            r = orc.lib.oracle_absmax_f32(fptr, n, nthr, ctypes.byref(used))
            ts.append(time.perf_counter() - t0)
        assert r == OUTLIER
        med = statistics.median(ts)
        cpu = {"value": round(nbytes / med / 1e9, 3), "unit": "GB/s", "cores": int(used.value),
               "kind": "port", "sample": f"the same 1e9-float buffer in host memory, median of {reps} full passes "
                                          "(OpenMP restatement of tests/side_aware.cu:216-219)"}

    peak, peak_kind = measured_peak()
    achieved = nbytes / (ms_per_step / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": profile_traffic("absmax_f32_1e9_side_aware"),
                "algorithmic_bytes_per_launch": nbytes,
                "kernel": "qrc_k_absmax_f32<1024>"}

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "n_per_gpu": n, "bytes_per_gpu": nbytes, "mode": args.mode,
                   "schedule": (args.sched if args.sched != "auto" else
                                "auto: " + ("static shares" if nbytes <= STATIC_MAX_BYTES else
                                            "balanced (static shares + queued tail)")),
                   "overlap": not args.no_overlap,
                   "launch": f"{info['num_sms_measured'] or ''} SMs x 1 CTA x 1024 threads",
                   "l2": L2_NOTE,
                   "parallelism": "replicated shards" if world == 1 else f"shard{world}+{collective}"},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "side_map": {k: info[k] for k in ("status_name", "mask", "chunk_bytes", "sms_side0", "sms_side1",
                                          "num_pages", "verify_probes", "verify_mismatches")},
        "init_ms": round(init_ms, 2),
        "ablation_gbs": ablation or None,
        "quant_e4m3": quant,
    }
    if world > 1:
        line["per_gpu_gbs"] = round(achieved, 2)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if px is not None:
        px.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    # Host-side OpenMP (data generation, CPU baselines): torchrun sets
    # OMP_NUM_THREADS=1 for its workers.  The reference arm runs alone on rank
    # 0 and takes every core; our ranks share the cores.  Set before any
    # OpenMP runtime is loaded.
    _, world, _ = dist_env()
    os.environ["OMP_NUM_THREADS"] = str(host_threads() if args.impl == "reference"
                                        else max(1, host_threads() // world))
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
