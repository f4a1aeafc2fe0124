"""ctypes binding of libqrc_b200.so (include/qrc_b200.h, include/qrc_b200_debug.h).

The library is loaded from quickruncuda_b200/lib/ only.  There is no fallback:
if the shared object is missing the import of this module raises, so nothing
can silently run a non-native path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "lib" / "libqrc_b200.so"
LIB_CHECKED_PATH = _PKG / "lib" / "libqrc_b200_checked.so"

c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_size = ctypes.c_size_t
c_int = ctypes.c_int
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p

QRC_OK = 0
QRC_ERR_INVALID = -1
QRC_ERR_CUDA = -2
QRC_ERR_DEVICE = -3
QRC_ERR_RANGE = -4
QRC_ERR_STATE = -5

MODE_SIDE_AWARE = 0
MODE_IGNORE_PAGE_BITS = 1
MODE_WRONG_SIDE = 2
MODE_STREAM = 3
OP_ABSMAX, OP_MAX, OP_MIN, OP_SUM, OP_SUMSQ = 0, 1, 2, 3, 4
OP_NAMES = {"absmax": OP_ABSMAX, "max": OP_MAX, "min": OP_MIN, "sum": OP_SUM, "sumsq": OP_SUMSQ}

SCHED_AUTO = 0x00
SCHED_STATIC = 0x10
SCHED_QUEUE = 0x20
SCHED_BALANCED = 0x30
SCHED_NAMES = {"auto": SCHED_AUTO, "static": SCHED_STATIC, "queue": SCHED_QUEUE, "balanced": SCHED_BALANCED}
MODE_NAMES = {"side_aware": MODE_SIDE_AWARE, "ignore_page_bits": MODE_IGNORE_PAGE_BITS,
              "random_side": MODE_IGNORE_PAGE_BITS, "wrong_side": MODE_WRONG_SIDE,
              "stream": MODE_STREAM}

SIDE_OK = 0
SIDE_NOT_RUN = 100


class SideInfo(ctypes.Structure):
    _fields_ = [(name, c_u32) for name in (
        "status", "mask", "mask_measured", "chunk_bytes", "num_sms_measured", "sms_side0",
        "sms_side1", "num_pages", "verify_probes", "verify_mismatches", "cal_lat_side0",
        "cal_lat_side1", "sm_lat_cluster0", "sm_lat_cluster1", "discover_smid", "reserved")]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_ if name != "reserved"}


# (name, restype, argtypes) for every entry point of the two headers.
SIGNATURES = [
    ("qrc_ctx_create", c_int, [ctypes.POINTER(c_void_p), c_int, c_void_p, c_size, c_void_p]),
    ("qrc_ctx_destroy", c_int, [c_void_p]),
    ("qrc_ctx_get_info", c_int, [c_void_p, ctypes.POINTER(SideInfo)]),
    ("qrc_ctx_set_mode", c_int, [c_void_p, c_int]),
    ("qrc_ctx_set_launch", c_int, [c_void_p, c_int, c_int]),
    ("qrc_ctx_set_pipeline", c_int, [c_void_p, c_int]),
    ("qrc_ctx_set_overlap", c_int, [c_void_p, c_int]),
    ("qrc_absmax_f32", c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p]),
    ("qrc_reduce_f32", c_int, [c_void_p, c_size, c_int, c_void_p, c_void_p, c_void_p]),
    ("qrc_alloc_like", c_int, [ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_void_p]),
    ("qrc_free_like", c_int, [c_void_p]),
    ("qrc_copy_f32", c_int, [c_void_p, c_void_p, c_size, c_void_p, c_void_p]),
    ("qrc_xchg_create", c_int, [ctypes.POINTER(c_void_p), c_int, c_int, c_int]),
    ("qrc_xchg_get_handle", c_int, [c_void_p, c_void_p]),
    ("qrc_xchg_set_peer", c_int, [c_void_p, c_int, c_void_p]),
    ("qrc_xchg_destroy", c_int, [c_void_p]),
    ("qrc_absmax_f32_allreduce", c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("qrc_xchg_debug_set_peer_ptr", c_int, [c_void_p, c_int, c_void_p]),
    ("qrc_xchg_debug_slots", c_void_p, [c_void_p]),
    ("qrc_ctx_debug_quant_side_aware", c_int, [c_void_p, c_int]),
    ("qrc_ctx_debug_quant_fused", c_int, [c_void_p, c_int]),
    ("qrc_debug_quant_launches", c_int, [c_void_p, c_void_p, c_size, c_void_p]),
    ("qrc_xchg_debug_post", c_int, [c_void_p, c_int, ctypes.c_uint32, ctypes.c_uint32]),
    ("qrc_xchg_epoch", ctypes.c_uint32, [c_void_p]),
    ("qrc_absmax_f32_noalloc", c_int, [c_void_p, c_size, c_void_p, c_void_p]),
    ("qrc_absmax_f32_host", c_int, [c_void_p, c_size, ctypes.POINTER(c_float), c_void_p, c_void_p]),
    ("qrc_host_reserve", c_int, [c_void_p, c_size]),
    ("qrc_amax_quant_e4m3", c_int, [c_void_p, c_size, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("qrc_fill_uniform_f32", c_int, [c_void_p, c_size, c_u64, c_u64, c_void_p]),
    ("qrc_fill_normal_f32", c_int, [c_void_p, c_size, c_u64, c_u64, c_float, c_void_p]),
    ("qrc_fill_normal_bf16", c_int, [c_void_p, c_size, c_u64, c_u64, c_float, c_void_p]),
    ("qrc_host_fill_uniform_f32", c_int, [c_void_p, c_size, c_u64, c_u64]),
    ("qrc_host_fill_normal_f32", c_int, [c_void_p, c_size, c_u64, c_u64, c_float]),
    ("qrc_outlier_index", c_u64, [c_u64, c_u64]),
    ("qrc_outlier_sign", c_int, [c_u64]),
    ("qrc_status_string", ctypes.c_char_p, [c_int]),
    ("qrc_side_status_string", ctypes.c_char_p, [c_u32]),
    ("qrc_last_cuda_error", c_int, []),
    ("qrc_version", c_int, []),
    # debug header
    ("qrc_ctx_read_map", c_int, [c_void_p, ctypes.POINTER(c_u32), c_size, ctypes.POINTER(c_size)]),
    ("qrc_ctx_clear_diagnostics", c_int, [c_void_p]),
    ("qrc_is_checked_build", c_int, []),
    ("qrc_ctx_map_device_ptr", c_void_p, [c_void_p]),
    ("qrc_debug_cvt_e4m3", c_int, [c_void_p, c_size, c_void_p, c_void_p]),
    ("qrc_debug_read_stream", c_int, [c_void_p, c_size, c_int, c_int, c_int, c_void_p, c_void_p]),
]


class QrcError(RuntimeError):
    def __init__(self, fn: str, code: int, lib=None):
        msg = f"{fn} failed with status {code}"
        if lib is not None:
            try:
                msg += f" ({lib.qrc_status_string(code).decode()})"
                if code == QRC_ERR_CUDA:
                    msg += f", cudaError {lib.qrc_last_cuda_error()}"
            except Exception:  # pragma: no cover - best effort message
                pass
        super().__init__(msg)
        self.code = code


def _bind(path: Path) -> ctypes.CDLL:
    if not path.exists():
        raise ImportError(
            f"{path} is not built; run `python -m quickruncuda_b200.build` "
            "(the CUDA library is required, there is no CPU fallback)")
    lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_libs: dict = {}


def load(checked: bool | None = None) -> ctypes.CDLL:
    """Load (once) the normal or the checked build.  `checked=None` follows
    the QRC_CHECKED environment variable."""
    if checked is None:
        checked = os.environ.get("QRC_CHECKED", "0") == "1"
    key = bool(checked)
    if key not in _libs:
        _libs[key] = _bind(LIB_CHECKED_PATH if key else LIB_PATH)
    return _libs[key]


def check(lib: ctypes.CDLL, fn: str, code: int) -> None:
    if code != QRC_OK:
        raise QrcError(fn, code, lib)
