"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product never imports it.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None

P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        _lib.or_row_bytes.restype = I64
        _lib.or_row_bytes.argtypes = [I32, I64]
        _lib.or_dequant_rows.argtypes = [I32, P, I64, I64, P]
        _lib.or_quant_q8k.argtypes = [P, I64, P]
        _lib.or_quant_q80.argtypes = [P, I64, P]
        _lib.or_qmatvec.argtypes = [I32, P, I64, I64, P, I32, P, I32, I32]
        _lib.or_argmax.restype = I64
        _lib.or_argmax.argtypes = [P, I64]
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def dequant(dtype: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    w = np.ascontiguousarray(w)
    assert lib().or_dequant_rows(dtype, _p(w), rows, cols, _p(out)) == 0
    return out


def quant_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(len(x) // 256 * 292, np.uint8)
    lib().or_quant_q8k(_p(x), len(x), _p(out))
    return out


def quant_q80(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(len(x) // 32 * 34, np.uint8)
    lib().or_quant_q80(_p(x), len(x), _p(out))
    return out


def qmatvec(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, *, order: int = 0,
            ksplit: int = 1) -> np.ndarray:
    """y[i, r]; order 0 = reference AVX2 lane order, 1 = device chunk order."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    w = np.ascontiguousarray(w)
    rc = lib().or_qmatvec(dtype, _p(w), rows, cols, _p(x), x.shape[0], _p(y), order, ksplit)
    assert rc == 0, rc
    return y


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().or_argmax(_p(v), len(v)))
