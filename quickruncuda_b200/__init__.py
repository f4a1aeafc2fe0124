"""quickruncuda_b200 -- B200-native L2-side-aware FP32 absmax (and fused
amax -> FP8 e4m3 quantize) behind QuickRunCUDA's kernel-file plugin ABI and a
plain C ABI (include/qrc_b200.h).

Layout:
  csrc/side_aware_b200.cu   drop-in kernel file (init + kernel), also the
                            device code of the C-ABI library
  csrc/qrc_abi.cu           libqrc_b200.so: contexts, launches, quantize, generators
  harness/qrc_harness.cpp   C++ harness running kernel files like QuickRunCUDA
  api.py / _native.py       Python binding of the C ABI (ctypes)
  build.py                  in-tree nvcc build (sm_100a)
"""
from pathlib import Path

from ._native import (MODE_IGNORE_PAGE_BITS, MODE_SIDE_AWARE, MODE_STREAM, MODE_WRONG_SIDE,
                      QrcError, load)
from .api import (SideAwareContext, fill_normal, fill_normal_bf16, fill_uniform, host_fill_normal,
                  host_fill_uniform, outlier)

PACKAGE_DIR = Path(__file__).resolve().parent
KERNEL_FILE = PACKAGE_DIR / "csrc" / "side_aware_b200.cu"
HARNESS = PACKAGE_DIR / "bin" / "qrc_harness"

__all__ = ["SideAwareContext", "fill_uniform", "fill_normal", "fill_normal_bf16", "host_fill_uniform",
           "host_fill_normal", "outlier", "load", "QrcError", "MODE_SIDE_AWARE", "MODE_IGNORE_PAGE_BITS",
           "MODE_WRONG_SIDE", "MODE_STREAM", "KERNEL_FILE", "HARNESS"]
