"""Build the native parts of quickruncuda_b200 in-tree.

Outputs (git-ignored, shipped with the source tree to the GPU machine):
  quickruncuda_b200/lib/libqrc_b200.so          C ABI of include/qrc_b200.h (sm_100a)
  quickruncuda_b200/lib/libqrc_b200_checked.so  same, with per-access bounds and
                                                coverage checks (test builds)
  quickruncuda_b200/bin/qrc_harness             C++ harness for kernel files

Run `python -m quickruncuda_b200.build` (or call build()).  Rebuilds only what
is older than its sources unless force=True.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB_DIR = PKG / "lib"
BIN_DIR = PKG / "bin"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_COMMON = GENCODE + ["-lineinfo", "-O3", "--std=c++17", "-Xptxas", "-v",
                         "-Xcompiler", "-fPIC,-fopenmp,-fvisibility=hidden"]

LIB_SOURCES = [CSRC / "qrc_abi.cu", CSRC / "qrc_noalloc.cu", CSRC / "side_aware_b200.cu", CSRC / "qrc_gen.cuh",
               INCLUDE / "qrc_b200.h", INCLUDE / "qrc_b200_debug.h"]
HARNESS_SOURCES = [PKG / "harness" / "qrc_harness.cpp", CSRC / "qrc_gen.cuh"]

LIB_PATH = LIB_DIR / "libqrc_b200.so"
LIB_CHECKED_PATH = LIB_DIR / "libqrc_b200_checked.so"
HARNESS_PATH = BIN_DIR / "qrc_harness"
KERNEL_FILE = CSRC / "side_aware_b200.cu"


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def _run(cmd, log: Path | None = None, verbose: bool = False) -> str:
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if log is not None:
        log.write_text(" ".join(cmd) + "\n" + res.stdout)
    if res.returncode != 0:
        sys.stderr.write(res.stdout)
        raise RuntimeError(f"build step failed ({res.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stdout.write(res.stdout)
    return res.stdout


def build_lib(checked: bool = False, force: bool = False, verbose: bool = False) -> Path:
    out = LIB_CHECKED_PATH if checked else LIB_PATH
    if not force and not _stale(out, LIB_SOURCES):
        return out
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = [NVCC, *NVCC_COMMON, "-shared", "-o", str(tmp), str(CSRC / "qrc_abi.cu"), str(CSRC / "qrc_noalloc.cu"),
           "-lgomp"]
    if checked:
        cmd.insert(1, "-DQRC_CHECKED")
    _run(cmd, log=LIB_DIR / (out.name + ".buildlog"), verbose=verbose)
    os.replace(tmp, out)
    return out


def build_harness(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale(HARNESS_PATH, HARNESS_SOURCES):
        return HARNESS_PATH
    BIN_DIR.mkdir(parents=True, exist_ok=True)
    cxx = shutil.which("g++") or "g++"
    tmp = HARNESS_PATH.with_name(HARNESS_PATH.name + ".tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fopenmp", f"-I{CUDA_HOME}/include",
           "-o", str(tmp), str(PKG / "harness" / "qrc_harness.cpp"),
           f"-L{CUDA_HOME}/lib64", "-lnvrtc", "-ldl", f"-Wl,-rpath,{CUDA_HOME}/lib64"]
    _run(cmd, log=BIN_DIR / "qrc_harness.buildlog", verbose=verbose)
    os.replace(tmp, HARNESS_PATH)
    return HARNESS_PATH


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(checked=False, force=force, verbose=verbose)
    build_lib(checked=True, force=force, verbose=verbose)
    build_harness(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH, LIB_CHECKED_PATH, HARNESS_PATH)
