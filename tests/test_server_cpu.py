"""Harness server mode without a GPU (compile-only commands): the FIFO
protocol of the reference's server (QuickRunCUDA.cpp:298-343,
utils/ipc_helper.h), quoting, error answers that leave the server running,
and a clean exit that removes the FIFOs."""
import os

from quickruncuda_b200 import KERNEL_FILE
from quickruncuda_b200.cuda_controller import CUDAController


def test_server_compiles_answers_errors_and_exits(tmp_path):
    c = CUDAController(server_dir=str(tmp_path))
    try:
        r = c.send_command(["--compile-only", "--arch", "sm_100a", KERNEL_FILE])
        assert r.startswith("compiled ") and "sm_100a" in r
        r = c.send_command(["--bogus-option"])
        assert r == "error: unknown option --bogus-option\n"
        r = c.send_command(["--clock-speed", "1500", KERNEL_FILE])
        assert "not supported" in r
        # a quoted header with spaces reaches NVRTC as one argument
        r = c.send_command(["-H", "#define QRC_PLUGIN_OP 3", "--compile-only", KERNEL_FILE])
        assert r.startswith("compiled ")
        r = c.send_command(["-H", "#define QRC_NO_SUCH_MACRO (", "--compile-only", KERNEL_FILE])
        assert r.startswith("compiled ")                       # an unused bad macro still compiles
        assert "qrc_harness" in c.send_command(["--help"])
    finally:
        assert c.close() == 0
    assert not os.path.exists(tmp_path / "quickruncuda_cmd")
    assert not os.path.exists(tmp_path / "quickruncuda_resp")
