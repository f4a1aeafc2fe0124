"""The C-ABI library and the harness on a machine without a GPU: the shared
objects load, export every declared symbol, the host-side generators agree
with the oracle bit for bit, and NVRTC compiles the drop-in kernel file with
the reference harness' options."""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))
KERNEL_FILE = ROOT / "quickruncuda_b200" / "csrc" / "side_aware_b200.cu"
HARNESS = ROOT / "quickruncuda_b200" / "bin" / "qrc_harness"


def declared_functions():
    names = []
    decl = re.compile(r"^(?:const\s+)?(?:struct\s+)?[A-Za-z_][\w]*[\s\*]+(qrc_\w+)\s*\(", re.M)
    for h in HEADERS:
        names += decl.findall(h.read_text())
    return sorted(set(names))


def test_headers_declare_the_entry_points():
    names = declared_functions()
    for must in ("qrc_ctx_create", "qrc_absmax_f32", "qrc_amax_quant_e4m3", "qrc_absmax_f32_host"):
        assert must in names


@pytest.mark.parametrize("checked", [False, True])
def test_library_exports_every_declared_symbol(checked):
    from quickruncuda_b200 import _native
    path = _native.LIB_CHECKED_PATH if checked else _native.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    lib = _native.load(checked)
    assert lib.qrc_is_checked_build() == int(checked)


def test_binding_covers_every_declared_symbol():
    from quickruncuda_b200 import _native
    bound = {name for name, _, _ in _native.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_status_strings(lib):
    assert lib.qrc_status_string(0) == b"ok"
    assert b"invalid" in lib.qrc_status_string(-1)
    assert lib.qrc_side_status_string(0) == b"side-aware"
    assert lib.qrc_version() >= 10000


def test_invalid_arguments_rejected_without_gpu(lib):
    # Argument checks come before any CUDA call.
    assert lib.qrc_absmax_f32(None, 16, None, None, None) == -1
    assert lib.qrc_ctx_create(None, 0, None, 0, None) == -1
    assert lib.qrc_ctx_set_mode(None, 0) == -1
    assert lib.qrc_reduce_f32(None, 16, 3, None, None, None) == -1
    assert lib.qrc_xchg_create(None, 0, 0, 1) == -1
    assert lib.qrc_alloc_like(None, None, None) == -1
    assert lib.qrc_copy_f32(None, None, 16, None, None) == -1
    assert lib.qrc_free_like(None) == 0
    assert lib.qrc_absmax_f32_allreduce(None, 16, None, None, None, None) == -1
    assert lib.qrc_ctx_destroy(None) == 0


@pytest.mark.parametrize("seed,offset", [(0, 0), (1, 0), (4, 3_000_000_000), (77, 12345)])
def test_host_generators_match_oracle(qrc, oracle, seed, offset):
    n = 100_003
    x = np.empty(n, np.float32)
    qrc.host_fill_uniform(x, seed, offset)
    assert np.array_equal(x.view(np.uint32), oracle.uniform(seed, n, offset).view(np.uint32))
    y = np.empty(n, np.float32)
    qrc.host_fill_normal(y, seed, 2.0, offset)
    assert np.array_equal(y.view(np.uint32), oracle.normal(seed, n, 2.0, offset).view(np.uint32))


@pytest.mark.parametrize("seed,n", [(0, 1048576), (1, 1_000_000_000), (4, 8_000_000_000), (9, 1)])
def test_outlier_placement_matches_oracle(qrc, oracle, seed, n):
    assert qrc.outlier(seed, n) == oracle.outlier(seed, n)


def _harness(*args, check=True):
    return subprocess.run([str(HARNESS), *map(str, args)], capture_output=True, text=True, check=check)


@pytest.mark.parametrize("arch", ["sm_100a", "sm_100"])
@pytest.mark.parametrize("header", ["", "#define FORCE_RANDOM_SIDE", "#define FORCE_WRONG_SIDE",
                                    "#define QRC_PLUGIN_OP 2", "#define QRC_PLUGIN_OP 4"])
def test_kernel_file_compiles_with_nvrtc(arch, header):
    # The reference harness compiles kernel files with NVRTC, fast math and
    # C++17 for sm_100 on B200 (utils/cuda_helper.h:223-253); ours defaults to sm_100a.
    r = _harness("--compile-only", "--arch", arch, "-H", header, KERNEL_FILE)
    assert "compiled" in r.stdout


def test_harness_refuses_gpu_settings():
    r = _harness("--clock-speed", "1500", KERNEL_FILE, check=False)
    assert r.returncode != 0 and "not supported" in r.stderr
    r = _harness("--help")
    assert "--timedRuns" in r.stdout and "--fill-a" in r.stdout


def test_harness_unknown_option():
    r = _harness("--no-such-flag", check=False)
    assert r.returncode == 2


def test_kernel_file_is_self_contained():
    src = KERNEL_FILE.read_text()
    assert "#include" not in src.split("#ifndef QRC_SIDE_AWARE_B200_CU")[1]
    assert 'extern "C" __global__' in src and "init(" in src and "kernel(" in src


def _kernel_define(name):
    m = re.search(rf"^#define {name} (.+)$", KERNEL_FILE.read_text(), re.M)
    assert m, name
    return m.group(1).strip()


def test_bench_schedule_label_matches_kernel_threshold():
    """bench.py labels the automatic schedule by size; its byte threshold is
    the kernel's QRC_STATIC_MAX_PAIRS 8 KiB pairs."""
    import sys
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.STATIC_MAX_BYTES == int(_kernel_define("QRC_STATIC_MAX_PAIRS")) * 8192


def test_schedule_thresholds_are_ordered():
    """SM-first shares stay inside the static-only range, and the 1/8 static
    part applies only where the balanced schedule runs."""
    sm_first = int(_kernel_define("QRC_SM_FIRST_MAX_PAIRS"))
    static_max = int(_kernel_define("QRC_STATIC_MAX_PAIRS"))
    large = int(_kernel_define("QRC_LARGE_PAIRS"))
    plain = _kernel_define("QRC_PLAIN_MAX_BYTES")
    m = re.fullmatch(r"\((\d+)ull << 20\)", plain)
    assert m, plain
    assert sm_first <= static_max < large
    assert int(m.group(1)) << 20 <= static_max * 8192
    assert 0 <= int(_kernel_define("QRC_STATIC_EIGHTHS_LARGE")) <= int(_kernel_define("QRC_STATIC_EIGHTHS")) <= 8
