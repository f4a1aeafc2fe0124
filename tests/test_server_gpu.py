"""Harness server mode on a B200: several runs in one process (the context
stays alive), an error between them, and results equal to one-shot runs."""
import json

import numpy as np
import pytest

from quickruncuda_b200 import KERNEL_FILE
from quickruncuda_b200.cuda_controller import CUDAController

pytestmark = pytest.mark.gpu


def test_server_runs_kernel_files_back_to_back(tmp_path, oracle):
    n = 1 << 21
    base = ["-i", "-p", "-t", "1024", "-A", n, "-0", n, "-C", 1, "-T", 5, "--json"]
    with CUDAController(server_dir=str(tmp_path)) as c:
        for seed, op in [(0, 0), (1, 1), (2, 0)]:
            r = c.send_command(base + ["--fill-a", f"uniform:{seed}:7.5", "-H", f"#define QRC_PLUGIN_OP {op}",
                                       KERNEL_FILE])
            res = json.loads(r.strip().splitlines()[-1])
            host = oracle.uniform_with_outlier(seed, n, 7.5)
            want = oracle.absmax(host) if op == 0 else oracle.reduce("max", host)
            assert res["c0_bits"] == int(np.array([want], np.float32).view(np.uint32)[0]), (seed, op)
            assert res["avg_ms"] > 0
            r = c.send_command(["--cubin", str(tmp_path / "missing.cubin"), "-A", 16])
            assert r.startswith("error: cannot open")
