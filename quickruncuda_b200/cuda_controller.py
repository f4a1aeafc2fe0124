"""Python client of the harness' server mode, for fast sweeps: one harness
process keeps its CUDA context and runs command lines sent to it, so a sweep
pays no process start, driver load or context creation per point.

Mirrors the reference's utils/cuda_controller.py (class CUDAController,
send_command) and its FIFO protocol (utils/ipc_helper.h): a command line is
written to <dir>/quickruncuda_cmd, and the command's standard output comes
back on <dir>/quickruncuda_resp.  Unlike the reference, the FIFO directory can
be chosen (several servers can run side by side), and a failing command
answers with its error message ("error: ...") while the server keeps running.
"""
from __future__ import annotations

import os
import subprocess
import time
from pathlib import Path
from typing import Optional, Sequence

HARNESS = Path(__file__).resolve().parent / "bin" / "qrc_harness"


class CUDAController:
    def __init__(self, server_dir: Optional[str] = None, harness: Optional[str] = None, device: int = 0,
                 start_timeout: float = 30.0):
        self.server_dir = str(server_dir or "/tmp")
        self.cmd_pipe_path = os.path.join(self.server_dir, "quickruncuda_cmd")
        self.resp_pipe_path = os.path.join(self.server_dir, "quickruncuda_resp")
        args = [str(harness or HARNESS), "--server", "--server-dir", self.server_dir, "--device", str(device)]
        self.process = subprocess.Popen(args, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE)
        t0 = time.monotonic()
        while not (os.path.exists(self.cmd_pipe_path) and os.path.exists(self.resp_pipe_path)):
            if self.process.poll() is not None:
                raise RuntimeError(f"harness server exited: {self.process.stderr.read().decode()}")
            if time.monotonic() - t0 > start_timeout:
                self.process.kill()
                raise TimeoutError("harness server did not create its FIFOs")
            time.sleep(0.05)

    def send_command(self, args: Sequence, read_response: bool = True) -> Optional[str]:
        """Runs one harness command line in the server; returns its output.
        Arguments containing spaces are quoted with '...' as the reference
        parser expects."""
        cmd = " ".join(f"'{a}'" if " " in str(a) else str(a) for a in args)
        with open(self.cmd_pipe_path, "w") as f:
            f.write(cmd)
        if not read_response:
            return None
        with open(self.resp_pipe_path, "r") as f:
            return f.read()

    def close(self, timeout: float = 30.0) -> int:
        """Sends "exit" and waits for the server; returns its exit status."""
        if self.process.poll() is None:
            self.send_command(["exit"], read_response=False)
            try:
                self.process.wait(timeout=timeout)
            except subprocess.TimeoutExpired:
                self.process.kill()
                self.process.wait()
        return self.process.returncode

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            if getattr(self, "process", None) is not None and self.process.poll() is None:
                self.close()
        except Exception:
            pass
