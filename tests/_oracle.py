"""ctypes binding of the CPU oracle (oracle/liboracle.so) for the tests.

The oracle is the checker: tests compare the CUDA path with it; nothing in the
product imports this module.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
ORACLE_DIR = ROOT / "oracle"
ORACLE_SO = ORACLE_DIR / "liboracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class Oracle:
    def __init__(self, lib: ctypes.CDLL):
        self.lib = lib
        L = lib
        u64, sz, f32, i32, u32 = ctypes.c_uint64, ctypes.c_size_t, ctypes.c_float, ctypes.c_int, ctypes.c_uint32
        for name, res, args in [
            ("oracle_splitmix64", u64, [u64, u64, ctypes.c_uint]),
            ("oracle_fill_uniform", None, [u64, u64, sz, _f32p]),
            ("oracle_fill_normal", None, [u64, u64, sz, f32, _f32p]),
            ("oracle_fill_normal_bf16", None, [u64, u64, sz, f32, _u16p]),
            ("oracle_f32_to_bf16", ctypes.c_uint16, [f32]),
            ("oracle_bf16_to_f32", f32, [ctypes.c_uint16]),
            ("oracle_outlier_index", u64, [u64, u64]),
            ("oracle_outlier_sign", i32, [u64]),
            ("oracle_absmax_f32_serial", f32, [_f32p, sz]),
            ("oracle_absmax_f32", f32, [_f32p, sz, i32, ctypes.POINTER(i32)]),
            ("oracle_absmax_bf16", f32, [_u16p, sz]),
            ("oracle_max_f32", f32, [_f32p, sz]),
            ("oracle_min_f32", f32, [_f32p, sz]),
            ("oracle_sum_f32", ctypes.c_double, [_f32p, sz, ctypes.POINTER(ctypes.c_double)]),
            ("oracle_sumsq_f32", ctypes.c_double, [_f32p, sz, ctypes.POINTER(ctypes.c_double)]),
            ("oracle_f32_to_e4m3", ctypes.c_uint8, [f32]),
            ("oracle_e4m3_to_f32", f32, [ctypes.c_uint8]),
            ("oracle_f32_bits_to_e4m3", None, [u32, sz, _u8p]),
            ("oracle_e4m3_scale", f32, [f32]),
            ("oracle_amax_quant_e4m3", f32, [_u16p, sz, _u8p]),
            ("oracle_pair_half", i32, [u64, u32, i32, i32]),
            ("oracle_fill_ref_random", None, [ctypes.c_uint, ctypes.c_uint, sz, _u32p]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args

    @classmethod
    def load(cls) -> "Oracle":
        srcs = [ORACLE_DIR / "oracle.c", ORACLE_DIR / "oracle_mt.cpp"]
        if not ORACLE_SO.exists() or any(s.stat().st_mtime > ORACLE_SO.stat().st_mtime for s in srcs):
            subprocess.run(["make", "-C", str(ORACLE_DIR), "oracle"], check=True,
                           stdout=subprocess.DEVNULL)
        return cls(ctypes.CDLL(str(ORACLE_SO)))

    # -- generators ----------------------------------------------------------
    def uniform(self, seed: int, n: int, offset: int = 0) -> np.ndarray:
        x = np.empty(n, np.float32)
        self.lib.oracle_fill_uniform(seed, offset, n, _p(x, _f32p))
        return x

    def normal(self, seed: int, n: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
        x = np.empty(n, np.float32)
        self.lib.oracle_fill_normal(seed, offset, n, sigma, _p(x, _f32p))
        return x

    def normal_bf16(self, seed: int, n: int, sigma: float = 1.0, offset: int = 0) -> np.ndarray:
        x = np.empty(n, np.uint16)
        self.lib.oracle_fill_normal_bf16(seed, offset, n, sigma, _p(x, _u16p))
        return x

    def outlier(self, seed: int, n: int) -> tuple[int, int]:
        return int(self.lib.oracle_outlier_index(seed, n)), int(self.lib.oracle_outlier_sign(seed))

    def uniform_with_outlier(self, seed: int, n: int, magnitude: float = 7.5) -> np.ndarray:
        x = self.uniform(seed, n)
        if n:
            i, s = self.outlier(seed, n)
            x[i] = np.float32(s * magnitude)
        return x

    def ref_random(self, seed: int, mask: int, n: int) -> np.ndarray:
        """The reference harness' `-r` fill of A (QuickRunCUDA.cpp:432-457)."""
        x = np.empty(n, np.uint32)
        self.lib.oracle_fill_ref_random(seed, mask, n, _p(x, _u32p))
        return x

    # -- reductions ------------------------------------------------------------
    def absmax(self, x: np.ndarray, threads: int = 0) -> np.float32:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return np.float32(self.lib.oracle_absmax_f32(_p(x, _f32p), x.size, threads, None))

    def absmax_bits(self, x: np.ndarray) -> int:
        return int(np.array([self.absmax(x)], np.float32).view(np.uint32)[0])

    def absmax_serial(self, x: np.ndarray) -> np.float32:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return np.float32(self.lib.oracle_absmax_f32_serial(_p(x, _f32p), x.size))

    def reduce(self, op: str, x: np.ndarray):
        """op in absmax/max/min (np.float32 result) or sum/sumsq (returns
        (float result, sum of |term|) for the error bound)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if op == "absmax":
            return self.absmax(x)
        if op in ("max", "min"):
            return np.float32(getattr(self.lib, f"oracle_{op}_f32")(_p(x, _f32p), x.size))
        a = ctypes.c_double()
        r = getattr(self.lib, f"oracle_{op}_f32")(_p(x, _f32p), x.size, ctypes.byref(a))
        return float(r), float(a.value)

    def absmax_bf16(self, x: np.ndarray) -> np.float32:
        x = np.ascontiguousarray(x, dtype=np.uint16)
        return np.float32(self.lib.oracle_absmax_bf16(_p(x, _u16p), x.size))

    # -- e4m3 --------------------------------------------------------------------
    def e4m3(self, x: float) -> int:
        return int(self.lib.oracle_f32_to_e4m3(float(x)))

    def e4m3_decode(self, c: int) -> float:
        return float(self.lib.oracle_e4m3_to_f32(c))

    def e4m3_bits_range(self, first_bits: int, n: int) -> np.ndarray:
        out = np.empty(n, np.uint8)
        self.lib.oracle_f32_bits_to_e4m3(first_bits, n, _p(out, _u8p))
        return out

    def scale(self, amax: float) -> np.float32:
        return np.float32(self.lib.oracle_e4m3_scale(float(amax)))

    def amax_quant_e4m3(self, x_bf16: np.ndarray) -> tuple[np.ndarray, np.float32]:
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        q = np.empty(x.size, np.uint8)
        s = self.lib.oracle_amax_quant_e4m3(_p(x, _u16p), x.size, _p(q, _u8p))
        return q, np.float32(s)

    def pair_half(self, pair_addr: int, mask: int, page_bit: int, side: int) -> int:
        return int(self.lib.oracle_pair_half(pair_addr, mask, page_bit, side))
