"""The drop-in boundary on the GPU: the kernel file runs under our harness
(NVRTC, sm_100a and sm_100) and under the reference harness itself (built from
its sources into oracle/_ref/), with results equal to the oracle; the
reference kernel (also built from its sources) runs under our harness on the
same data."""
import json
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
KERNEL_FILE = ROOT / "quickruncuda_b200" / "csrc" / "side_aware_b200.cu"
HARNESS = ROOT / "quickruncuda_b200" / "bin" / "qrc_harness"
REF_DIR = ROOT / "oracle" / "_ref"
REF_HARNESS = REF_DIR / "QuickRunCUDA"
REF_CUBIN = REF_DIR / "side_aware_ref.cubin"
REF_CUBIN_999 = REF_DIR / "side_aware_ref_999.cubin"


def run(cmd, cwd, check=True, timeout=600):
    r = subprocess.run([str(c) for c in cmd], cwd=cwd, capture_output=True, text=True, timeout=timeout)
    if check and r.returncode != 0:
        raise AssertionError(f"{cmd} -> {r.returncode}\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}")
    return r


def c0_bits(path: Path) -> int:
    return int(np.fromfile(path, dtype=np.uint32)[0])


def harness_json(args, cwd):
    r = run([HARNESS, *args, "--json"], cwd)
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("arch", ["sm_100a", "sm_100"])
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 16, 32, 48])
def test_kernel_file_under_our_harness_config1(tmp_path, oracle, arch, mode):
    n = 1048576
    res = harness_json(["-i", "-p", "-t", "1024", "-A", 4 * n, "-0", n, "-1", mode, "-C", 1, "-T", 5,
                        "-P", 4 * n / 1e9, "-U", "GB/s", "--arch", arch, "--fill-a", "uniform:0:7.5",
                        KERNEL_FILE], tmp_path)
    assert res["c0"] == 7.5
    assert res["c0_bits"] == oracle.absmax_bits(oracle.uniform_with_outlier(0, n, 7.5))


@pytest.mark.parametrize("n", [1, 3, 5, 1023, 4096, 8193, (1 << 21) + 5, 3 * (1 << 20) - 1])
def test_kernel_file_odd_sizes_under_our_harness(tmp_path, oracle, n):
    # -A larger than -0: the kernel reads only the first n floats.
    res = harness_json(["-i", "-p", "-t", "1024", "-A", max(4 * n, 1 << 21), "-0", n, "-C", 1, "-T", 3,
                        "--fill-a", "uniform:13:3.25", KERNEL_FILE], tmp_path)
    full = oracle.uniform_with_outlier(13, max(4 * n, 1 << 21), 3.25)
    assert res["c0_bits"] == oracle.absmax_bits(full[:n])


def test_reference_c_compare_and_exit_status(tmp_path, oracle):
    n = 1 << 20
    want = np.array([oracle.absmax(oracle.uniform(7, n))], np.float32)
    good, bad = tmp_path / "good.bin", tmp_path / "bad.bin"
    want.tofile(good)
    (want * 2).tofile(bad)
    base = ["-i", "-p", "-t", "1024", "-A", n, "-0", n, "-C", 1, "-T", 2, "--fill-a", "uniform:7", KERNEL_FILE]
    assert run([HARNESS, *base, "--reference-c", good], tmp_path).returncode == 0
    r = run([HARNESS, *base, "--reference-c", bad], tmp_path, check=False)
    assert r.returncode == 1 and "First difference" in r.stdout


def test_report_line_format(tmp_path):
    n = 1 << 22
    r = run([HARNESS, "-i", "-p", "-t", "1024", "-A", n, "-0", n, "-T", 10, "-P", 4 * n / 1e9, "-U", "GB/s",
             "-L", "6547.8", "--fill-a", "uniform:1", KERNEL_FILE], tmp_path)
    line = [l for l in r.stdout.splitlines() if " ms ==> " in l][0]
    parts = line.split(" ==> ")
    assert parts[0].endswith(" ms") and parts[1].endswith(" GB/s") and parts[2].endswith("%")


needs_ref = pytest.mark.skipif(not REF_HARNESS.exists() or not REF_CUBIN.exists(),
                               reason="reference artefacts not built (oracle/_ref)")


@needs_ref
@pytest.mark.parametrize("seed,mask,n", [(1234, 0x3FFFFFFF, 1 << 20), (7, 0xBF7FFFFF, (1 << 22) + 4),
                                         (99, 0xFFFFFFFF, 5_000_000)])
def test_kernel_file_under_reference_harness(tmp_path, oracle, seed, mask, n):
    """Drop-in: the reference's own harness (NVRTC, sm_100, fast math) runs our
    kernel file on its `-r` data; C[0] equals the oracle on the identical fill."""
    out = tmp_path / "c.bin"
    run([REF_HARNESS, "-i", "-p", "-t", "1024", "-A", n, "-0", n, "-C", 1, "-T", 5, "-P", 4 * n / 1e9,
         "-U", "GB/s", "-r", "--randomSeed", seed, "--randomMask", hex(mask), "--dump-c", out,
         KERNEL_FILE], tmp_path)
    x = oracle.ref_random(seed, mask, n).view(np.float32)
    assert c0_bits(out) == oracle.absmax_bits(x)


@needs_ref
def test_reference_kernel_under_our_harness(tmp_path, oracle):
    """The reference kernel on a 1 Mi-float uniform input with one planted 7.5
    gives the oracle's answer."""
    n = 1048576
    res = harness_json(["--cubin", REF_CUBIN, "-i", "-p", "-t", "1024", "-A", 4 * n, "-0", n, "-C", 1,
                        "-T", 3, "--fill-a", "uniform:0:7.5"], tmp_path)
    assert res["c0"] == 7.5


@needs_ref
def test_reference_known_answer_999(tmp_path):
    """The reference's DEBUG_STORE_999_IN_A hook (tests/side_aware.cu:199-203)."""
    n = 1 << 22
    res = harness_json(["--cubin", REF_CUBIN_999, "-i", "-p", "-t", "1024", "-A", n, "-0", n, "-C", 1,
                        "-T", 2, "--fill-a", "uniform:2"], tmp_path)
    assert res["c0"] == 999.0


def test_kernel_file_at_the_plugin_int_limit(tmp_path):
    """n = 2^31 - 1 floats (8.6 GB), the largest `-0` the plugin's int
    argument can carry (tests/side_aware.cu:257): the planted outlier is the
    result."""
    n = (1 << 31) - 1
    res = harness_json(["-i", "-p", "-t", "1024", "-A", n, "-0", n, "-C", 1, "-T", 2,
                        "--fill-a", "uniform:5:7.5", KERNEL_FILE], tmp_path)
    assert res["c0"] == 7.5
