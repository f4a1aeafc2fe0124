"""Benchmark of the side-aware FP32 absmax on B200 (one JSON line on stdout).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1: the 1e9-float workload (4 GB, uniform[-1,1) from seed 1, one outlier of
magnitude 7.5 at a seeded index).  A step is one reduction of the whole
buffer: one kernel launch through the C ABI (qrc_absmax_f32).
N > 1 (one process per GPU under torchrun): every rank holds 1e9 floats of the
seed-4 uniform stream (rank r: elements [r*1e9, (r+1)*1e9)), one global
outlier on a seeded rank; a step is the per-shard reduction whose last CTA
also takes the maximum over the ranks (NVLink peer stores), or the reduction
plus an NCCL max all-reduce (--collective nccl).  Weak scaling.

`value` is whole-job GB/s with inputs resident in HBM (the 4 GB input is 32x
the 126 MB L2, so no flush is needed between steps).  `e2e` is the same metric
through qrc_absmax_f32_host: every step copies the 4 GB shard from pinned host
memory and reads the 4-byte result back.  `--impl reference` times the CPU
restatement of the reference reduction (oracle/, OpenMP on all host cores),
since the reference has no CPU implementation of this path.

Besides the headline, rank 0 at N = 1 reports (outside the timed region):
  ablation_gbs      every read mode under every work schedule
  roofline          achieved / measured copy peak, plus a measured read-only
                    ceiling (a plain streaming read at several depths)
  power             absmax of 1e9 normal(0,1) floats, seed 2: time-based runs of
                    side-aware, page-bits-ignored and plain-stream reads with
                    NVML energy per byte
  reference_kernel  the reference's own kernel (built from its source into
                    oracle/_ref/) and this kernel file, both under the C++
                    harness in stream order, on the same 1e9-float input
  quant_e4m3        the fused amax -> e4m3 quantize of a bf16 [16384, 8192]
                    normal(0,2) tensor, seed 3
At N > 1 every rank's step time, the reduction alone and the NCCL variant are
timed back to back, so the exchange's cost and the rank skew are visible.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_PER_GPU = 1_000_000_000
OUTLIER = 7.5
METRIC = "FP32 absmax GB/s at 1e9 floats (% of B200 HBM peak) at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
# HBM3e pin rate of a B200: 8 stacks x 1024 bits x 2 x 3996 MHz.
HBM_PIN_GBS = 8 * 1024 * 2 * 3996e6 / 8 / 1e9
# The kernel's automatic schedule: static per-SM shares alone up to this many
# input bytes (32,768 pairs of 8 KiB), static shares with a queued tail above.
STATIC_MAX_BYTES = 32768 * 8192
L2_NOTE = "input 4 GB per GPU > 126 MB L2 (no flush needed)"
TRAFFIC_RECORD = ROOT / "profiles" / "absmax_f32_1e9_side_aware.traffic.json"
# The reduction's device code (the headline kernel instantiates it); the
# traffic record is stale once this file changes.
KERNEL_SOURCES = [ROOT / "quickruncuda_b200" / "csrc" / "side_aware_b200.cu"]
KERNEL_FILE = ROOT / "quickruncuda_b200" / "csrc" / "side_aware_b200.cu"
REF_CUBIN = ROOT / "oracle" / "_ref" / "side_aware_ref.cubin"
HARNESS = ROOT / "quickruncuda_b200" / "bin" / "qrc_harness"


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
    ap.add_argument("--no-power", action="store_true")
    ap.add_argument("--no-refkernel", action="store_true")
    ap.add_argument("--no-ceiling", action="store_true")
    ap.add_argument("--power-seconds", type=float, default=5.0, help="length of each time-based power run")
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


def workload(world: int, n: int) -> dict:
    """The `config` both arms print: the data, not how either arm runs it."""
    if world == 1:
        w = f"absmax of {n} f32 uniform[-1,1) seed 1 + one outlier 7.5 at a seeded index"
    else:
        w = f"sharded absmax: {world} x {n} f32 uniform[-1,1) seed 4, one global outlier 7.5, max all-reduce"
    return {"workload": w, "n_per_gpu": n, "bytes_per_gpu": 4 * n, "n_gpus": world, "l2": L2_NOTE}


def data_of(world: int, n: int, rank: int, outlier_fn):
    """(seed, element offset, local outlier index or None, sign) of `rank`'s shard."""
    if world == 1:
        seed, offset = 1, 0
        gi, sign = outlier_fn(seed, n)
    else:
        seed, offset = 4, rank * n
        gi, sign = outlier_fn(seed, world * n)
    local = gi - offset if offset <= gi < offset + n else None
    return seed, offset, local, sign


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def sources_sha() -> str:
    h = hashlib.sha256()
    for p in KERNEL_SOURCES:
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def traffic_record(n: int):
    """DRAM bytes per launch from the committed ncu record (read + write per
    launch, one capture of the full-size workload), with whether the kernel
    sources changed since that capture.  None when no record matches n."""
    if not TRAFFIC_RECORD.exists():
        return None, None
    rec = json.loads(TRAFFIC_RECORD.read_text())
    if int(rec.get("n", -1)) != n:
        return None, None
    total = int(rec["dram_bytes_read_per_launch"]) + int(rec["dram_bytes_write_per_launch"])
    meta = {"record": str(TRAFFIC_RECORD.relative_to(ROOT)), "captured": rec.get("captured"),
            "launches": rec.get("launches"), "sources_sha": rec.get("sources_sha"),
            "stale": rec.get("sources_sha") != sources_sha()}
    return total, meta


class ClockSampler:
    """NVML sampler (read-only) for the timed region: SM clock, power and
    clock-event reasons, plus the energy counter at both ends."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x10: "sync_boost", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.001):
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
        self.e0 = self.e1 = None

    def _reasons(self):
        nv = self.nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self.h))

    def energy_mj(self):
        try:
            return int(self.nv.nvmlDeviceGetTotalEnergyConsumption(self.h))
        except Exception:
            return None

    def sample(self):
        try:
            clk = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
            pw = self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
            self.samples.append((clk, pw, self._reasons()))
        except Exception:
            pass

    def _loop(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.e0 = self.energy_mj()
            self._th = threading.Thread(target=self._loop, daemon=True)
            self._th.start()
        return self

    def __exit__(self, *exc):
        if self._th:
            self._stop.set()
            self._th.join()
            self.sample()
            self.e1 = self.energy_mj()

    def energy_j(self):
        if self.e0 is None or self.e1 is None:
            return None
        return (self.e1 - self.e0) / 1e3

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
    from tests._oracle import Oracle
    orc = Oracle.load()
    n = args.n_per_gpu
    nbytes = 4 * n

    def outlier_fn(seed, total):
        return orc.outlier(seed, total)

    # The sample is one shard of the workload: at N = 1 the whole input; at
    # N > 1 the shard that holds the global outlier (the host cores are the
    # same whichever shard they read, so GB/s is the whole job's rate).
    sample_rank = 0
    if world > 1:
        gi, _ = outlier_fn(4, world * n)
        sample_rank = gi // n
    seed, offset, local, sign = data_of(world, n, sample_rank, outlier_fn)
    x = orc.uniform(seed, n, offset)
    if local is not None:
        x[local] = OUTLIER * sign
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
    sample = (f"the full {n}-float input" if world == 1 else
              f"shard {sample_rank} of {world} ({n} floats, the one holding the outlier)")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / len(times), 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload(world, n),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": int(used.value), "kind": "port",
                         "sample": f"{sample}, {args.steps} passes (OpenMP restatement of "
                                   "tests/side_aware.cu:216-219; the reference has no CPU path)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def timed(fn, steps, stream):
    """ms per call of `fn`, `steps` calls between two events on `stream`."""
    import torch
    s, e = _events()
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / steps


def read_ceiling(lib, x, nbytes, stream, dev):
    """Best GB/s of a plain streaming read of the same buffer (no side map,
    nothing computed but an XOR) over several in-flight depths and shapes."""
    import torch
    from quickruncuda_b200 import _native as nat
    sink = torch.zeros(4, dtype=torch.int32, device=dev)
    best, runs = 0.0, {}
    for depth, threads, blocks_per_sm in ((8, 1024, 1), (4, 1024, 2), (16, 512, 1), (32, 256, 1)):
        def go():
            nat.check(lib, "qrc_debug_read_stream",
                      lib.qrc_debug_read_stream(ctypes.c_void_p(x.data_ptr()), nbytes, depth, threads, blocks_per_sm,
                                                ctypes.c_void_p(sink.data_ptr()), ctypes.c_void_p(stream.cuda_stream)))
        for _ in range(3):
            go()
        ms = timed(go, 20, stream)
        gbs = nbytes / (ms / 1e3) / 1e9
        runs[f"depth{depth}_t{threads}x{blocks_per_sm}"] = round(gbs, 1)
        best = max(best, gbs)
    return round(best, 1), runs


def power_runs(q, ctx, x, out, stream, local, seconds):
    """Absmax of 1e9 normal(0,1) floats, seed 2.  Each variant runs back to back for
    `seconds` (twice, interleaved), with NVML energy and clocks sampled."""
    import torch
    n = x.numel()
    nbytes = 4 * n
    q.fill_normal(x, seed=2, sigma=1.0)
    torch.cuda.synchronize()
    variants = (("side_aware", "balanced"), ("ignore_page_bits", "balanced"), ("stream", "auto"))
    res = {f"{m}/{s}": [] for m, s in variants}
    bits = set()
    for _round in range(2):
        for m, sched in variants:
            ctx.mode = m
            ctx.schedule = sched
            for _ in range(5):
                ctx.absmax(x, out=out)
            torch.cuda.synchronize()
            launches = 0
            s, e = _events()
            with ClockSampler(local, period_s=0.05) as cs:
                s.record(stream)
                t0 = time.perf_counter()
                while time.perf_counter() - t0 < seconds:
                    for _ in range(64):
                        ctx.absmax(x, out=out)
                    launches += 64
                    torch.cuda.synchronize()
                e.record(stream)
                torch.cuda.synchronize()
            ms = s.elapsed_time(e)
            bits.add(int(out.view(torch.int32).item()))
            ej = cs.energy_j()
            summ = cs.summary()
            gb = nbytes * launches / 1e9
            res[f"{m}/{sched}"].append({
                "gbs": round(gb / (ms / 1e3), 1), "seconds": round(ms / 1e3, 2), "launches": launches,
                "mean_w": round(ej / (ms / 1e3), 1) if ej else None,
                "j_per_gb": round(ej / gb, 5) if ej else None,
                "sm_mhz": summ["sm_mhz"], "reasons": summ["reasons"]})
    ctx.mode = "side_aware"
    ctx.schedule = "auto"
    out_v = {}
    for k, runs in res.items():
        jg = [r["j_per_gb"] for r in runs if r["j_per_gb"]]
        out_v[k] = {"runs": runs,
                    "j_per_gb": round(statistics.mean(jg), 5) if jg else None,
                    "spread_pct": round(100 * (max(jg) - min(jg)) / statistics.mean(jg), 2) if jg else None,
                    "gbs": round(statistics.mean(r["gbs"] for r in runs), 1),
                    "mean_w": round(statistics.mean(r["mean_w"] for r in runs if r["mean_w"]), 1) if jg else None}
    sa, ig = out_v["side_aware/balanced"]["j_per_gb"], out_v["ignore_page_bits/balanced"]["j_per_gb"]
    return {"workload": "absmax of 1e9 f32 normal(0,1) seed 2", "seconds_per_run": seconds,
            "runs_per_variant": 2, "variants": out_v, "results_identical": len(bits) == 1,
            "side_aware_vs_ignore_page_bits_energy_pct": round(100 * (sa - ig) / ig, 2) if sa and ig else None}


def reference_kernel_leg(n, local, ours_gbs):
    """The reference's sm_100 kernel (tests/side_aware.cu built from its source
    by oracle/Makefile) and this kernel file, both launched by the C++ harness
    in stream order (-i -p -t 1024, 100 timed runs, as the reference is run),
    on the same synthetic 1e9-float input.  Separate processes, after the
    timed region."""
    if not (REF_CUBIN.exists() and HARNESS.exists()):
        return {"unavailable": "oracle/_ref/side_aware_ref.cubin or the harness is not built"}
    common = ["-i", "-p", "-t", "1024", "-C", "1", "-A", str(n), "-0", str(n), "-P", str(4 * n / 1e9), "-U", "GB/s",
              "--fill-a", "uniform:1:7.5", "--json", "-T", "100", "--device", str(local)]
    res = {}
    for name, extra in (("reference_kernel_harness", ["--cubin", str(REF_CUBIN)]),
                        ("our_kernel_file_harness", [str(KERNEL_FILE)])):
        try:
            with tempfile.TemporaryDirectory(prefix="qrc_harness_") as work:    # the harness writes output.cubin there
                p = subprocess.run([str(HARNESS), *common, *extra], capture_output=True, text=True, timeout=300,
                                   cwd=work)
            d = json.loads(p.stdout.strip().splitlines()[-1])
            res[name] = {"gbs": round(d["perf"], 1), "us_per_launch": round(1e3 * d["avg_ms"], 2),
                         "c0": d["c0"], "correct": d["c0"] == OUTLIER}
        except Exception as e:                        # reported, never fatal to the bench line
            res[name] = {"error": repr(e)[:200]}
    res["our_c_abi_gbs"] = round(ours_gbs, 1)
    res["command"] = "qrc_harness " + " ".join(common) + " [--cubin oracle/_ref/side_aware_ref.cubin | kernel file]"
    return res


def run_ours(args):
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
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    stream = torch.cuda.current_stream(dev)

    # ---- input shard, resident in HBM ----
    n = args.n_per_gpu
    nbytes = 4 * n
    x = torch.empty(n, dtype=torch.float32, device=dev)
    seed, offset, local_out, sign = data_of(world, n, rank, q.outlier)
    q.fill_uniform(x, seed, offset=offset)
    if local_out is not None:
        x[local_out] = OUTLIER * sign
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
    nccl_max = None
    if world > 1:
        from quickruncuda_b200.sharded import MaxAllReduce, PeerMax
        nccl_max = MaxAllReduce()
        if args.collective == "fused":
            px = PeerMax.try_create(ctx)            # None on every rank if peers cannot be mapped
    collective = ("in-kernel NVLink peer max" if px is not None else "nccl_max_allreduce") if world > 1 else None

    def step():
        if px is not None:
            px.absmax(x, out)
            return
        ctx.absmax(x, out=out)
        if world > 1:
            nccl_max.enqueue(out)

    def settle():
        """Host-side end of a batch of steps: waits for outstanding NCCL
        collectives under a deadline (raises if a rank is gone)."""
        if nccl_max is not None:
            nccl_max.wait_all()
        torch.cuda.synchronize()

    for _ in range(max(args.warmup, 3)):
        step()
    settle()
    if world > 1:
        dist.barrier()
    assert out.item() == OUTLIER, f"warm-up result {out.item()} != {OUTLIER}"

    start, end = _events()
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        settle()
        if world > 1:
            dist.barrier()
    ms = start.elapsed_time(end)
    assert out.item() == OUTLIER, f"timed result {out.item()} != {OUTLIER}"
    rank_ms = [ms]
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        rank_ms = [float(v.item()) for v in allt]
    ms_total = max(rank_ms)
    ms_per_step = ms_total / args.steps
    value = world * nbytes / (ms_per_step / 1e3) / 1e9

    # ---- N > 1: rank skew and what the exchange costs ----
    multi = None
    if world > 1:
        def max_over_ranks(v):
            t = torch.tensor([v], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        ksteps = max(3, min(args.steps, 200))
        for _ in range(3):                      # the first launch of a kernel also loads it
            ctx.absmax(x, out=out)
        torch.cuda.synchronize()
        dist.barrier()
        local_ms = max_over_ranks(timed(lambda: ctx.absmax(x, out=out), ksteps, stream))

        def nccl_step():
            ctx.absmax(x, out=out)
            nccl_max.enqueue(out)
        for _ in range(3):                      # the communicator is set up by its first collective
            nccl_step()
        nccl_max.wait_all()
        torch.cuda.synchronize()
        dist.barrier()
        nccl_ms = timed(nccl_step, ksteps, stream)
        nccl_max.wait_all()
        assert out.item() == OUTLIER
        nccl_ms = max_over_ranks(nccl_ms)
        fused_ms = None
        if px is not None:
            for _ in range(3):
                px.absmax(x, out)
            torch.cuda.synchronize()
            dist.barrier()
            fused_ms = max_over_ranks(timed(lambda: px.absmax(x, out), ksteps, stream))
            assert out.item() == OUTLIER
        multi = {"rank_ms_per_step": [round(v / args.steps, 5) for v in rank_ms],
                 "rank_spread_us": round(1e3 * (max(rank_ms) - min(rank_ms)) / args.steps, 2),
                 "reduction_only_ms_per_step": round(local_ms, 5),
                 "fused_ms_per_step": round(fused_ms, 5) if fused_ms else None,
                 "nccl_ms_per_step": round(nccl_ms, 5),
                 "fused_exchange_cost_us": round(1e3 * (fused_ms - local_ms), 2) if fused_ms else None,
                 "nccl_exchange_cost_us": round(1e3 * (nccl_ms - local_ms), 2),
                 "steps_each": ksteps}

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
                abl_ms = timed(lambda: ctx.absmax(x, out=out), abl_steps, stream)
                assert out.item() == OUTLIER
                gbs = round(nbytes / (abl_ms / 1e3) / 1e9, 2)
                if m == "stream":
                    ablation[m] = gbs
                else:
                    ablation.setdefault(m, {})[sched] = gbs
        ctx.mode = args.mode
        ctx.schedule = args.sched

    ceiling, ceiling_runs = (None, None)
    if not args.no_ceiling and world == 1:
        ceiling, ceiling_runs = read_ceiling(ctx.lib, x, nbytes, stream, dev)

    refk = None
    if not args.no_refkernel and world == 1 and n == N_PER_GPU:
        refk = reference_kernel_leg(n, local, value)

    power = None
    if not args.no_power and world == 1:
        power = power_runs(q, ctx, x, out, stream, local, args.power_seconds)

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
            cq.set_overlap(not args.no_overlap)
            for _ in range(3):
                cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax)
            qsteps = max(3, min(args.steps, 300))
            qms = timed(lambda: cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax), qsteps, stream)
            launches = cq.quant_launches(xq, qout)
            cq.set_quant_fused(False)                  # the two-launch path, for comparison
            for _ in range(3):
                cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax)
            qms2 = timed(lambda: cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax), qsteps, stream)
            cq.set_quant_fused(True)
            cq.amax_quant_e4m3(xq, q=qout, scale=qscale, amax=qamax)
        qbytes = 2 * 2 * nq + nq          # two reads of the bf16 input (amax, then quantize) + one e4m3 write
        qbound = 2 * nq + nq              # one read + one write
        qgbs = qbytes / (qms / 1e3) / 1e9
        peak, _ = measured_peak()
        quant = {"workload": "bf16 [16384, 8192] normal(0,2) seed 3 -> e4m3 + scale", "ms": round(qms, 5),
                 "gbs": round(qgbs, 2), "algorithmic_bytes": qbytes, "launches_per_step": launches,
                 "two_launch_ms": round(qms2, 5),
                 "roofline_frac": round(qgbs / peak, 4),
                 "frac_of_one_read_one_write_bound": round(qbound / (qms / 1e3) / 1e9 / peak, 4),
                 "scale": float(qscale.item()), "amax": float(qamax.item())}
        del xq, qout

    # ---- end to end through the host-buffer C-ABI call ----
    e2e = None
    h_ptr = None
    if not args.no_e2e:
        e2e_steps = args.e2e_steps or min(10, max(3, args.steps // 100))
        host = torch.empty(n, dtype=torch.float32, pin_memory=True)
        q.host_fill_uniform(host, seed, offset)
        if local_out is not None:
            host[local_out] = OUTLIER * sign
        res = ctypes.c_float()
        lib = ctx.lib
        nat.check(lib, "qrc_host_reserve", lib.qrc_host_reserve(ctx.handle, n))   # staging set up outside the timing

        def e2e_step():
            rc = lib.qrc_absmax_f32_host(ctypes.c_void_p(host.data_ptr()), n, ctypes.byref(res), ctx.handle,
                                         ctypes.c_void_p(stream.cuda_stream))
            nat.check(lib, "qrc_absmax_f32_host", rc)
            if world > 1:
                t = torch.tensor([res.value], dtype=torch.float32, device=dev)
                nccl_max.enqueue(t)
                nccl_max.wait_all()
                return float(t.item())
            return res.value

        r0 = e2e_step()
        assert r0 == OUTLIER, r0
        if world > 1:
            dist.barrier()
        s, e = _events()
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
               "path": "qrc_absmax_f32_host (pinned host -> device staging in chunks on a copy stream, "
                       "each chunk reduced as it lands -> 4-byte result -> host)"}
        h_ptr = host

    # ---- CPU baseline on the same host data (rank 0, N = 1 only) ----
    cpu = None
    if world == 1 and not args.no_cpu:
        from tests._oracle import Oracle
        orc = Oracle.load()
        if h_ptr is None:
            h_ptr = torch.empty(n, dtype=torch.float32)
            q.host_fill_uniform(h_ptr, seed, offset)
            if local_out is not None:
                h_ptr[local_out] = OUTLIER * sign
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
    traffic, traffic_meta = traffic_record(n)
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "peak_note": "copy peak (read + write bytes) of measured; a pure read stream can exceed it",
                "traffic": traffic, "traffic_meta": traffic_meta,
                "algorithmic_bytes_per_launch": nbytes,
                "read_ceiling": ceiling, "read_ceiling_runs": ceiling_runs,
                "frac_of_read_ceiling": round(achieved / ceiling, 4) if ceiling else None,
                "hbm_pin_rate": round(HBM_PIN_GBS, 1), "frac_of_pin_rate": round(achieved / HBM_PIN_GBS, 4),
                "kernel": "qrc_k_absmax_f32<1024>"}

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload(world, n),
        "run": {"mode": args.mode,
                "schedule": (args.sched if args.sched != "auto" else
                             "auto: " + ("static shares" if nbytes <= STATIC_MAX_BYTES else
                                         "balanced (static shares + queued tail)")),
                "overlap": not args.no_overlap,
                "launch": f"{info['num_sms_measured'] or ''} SMs x 1 CTA x 1024 threads",
                "parallelism": "one GPU" if world == 1 else f"shard{world}+{collective}"},
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "side_map": {k: info[k] for k in ("status_name", "mask", "chunk_bytes", "sms_side0", "sms_side1",
                                          "num_pages", "verify_probes", "verify_mismatches")},
        "init_ms": round(init_ms, 2),
        "ablation_gbs": ablation or None,
        "power": power,
        "reference_kernel": refk,
        "quant_e4m3": quant,
    }
    if world > 1:
        line["per_gpu_gbs"] = round(achieved, 2)
        line["multi_gpu"] = multi
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
