"""ctypes binding of libiq.so (the C ABI declared in include/iq.h).

The library is loaded from the package directory; there is no fallback.  A
missing or unloadable library raises immediately so no caller can silently
run a CPU path.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libiq.so"
HEADER = PKG.parent / "include" / "iq.h"

_lib = None


class IqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"libiq error {code}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; run `python -m inferq_b200.build`")
        _lib = ctypes.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def declared_symbols() -> list[str]:
    """Every function name include/iq.h declares."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(iq_[a-z0-9_]+)\s*\(", text)))


P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int


def _declare(L: ctypes.CDLL) -> None:
    sig = {
        "iq_last_error": (ctypes.c_char_p, []),
        "iq_version": (ctypes.c_char_p, []),
        "iq_matrix_create": (I32, [I32, P, I64, I64, I32, ctypes.POINTER(P)]),
        "iq_matrix_leading_rows": (I32, [P, I64, ctypes.POINTER(P)]),
        "iq_matrix_destroy": (None, [P]),
        "iq_matrix_shape": (I32, [P, ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I32)]),
        "iq_matrix_forward_rows": (I32, [P, P, I64, P]),
        "iq_matrix_forward_device": (I32, [P, P, I32, P, P]),
        "iq_matrix_forward_device_noalloc": (I32, [P, P, I32, P, P]),
        "iq_matrix_forward_wide": (I32, [P, P, I32, P, P]),
        "iq_matrix_status": (I32, [P]),
        "iq_qgemv": (I32, [I32, P, I64, I64, P, I32, P, P]),
        "iq_qgemv_ksplit": (I32, [I32, I64, I64]),
        "iq_matrix_dequantize": (I32, [P, P, I64, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def check(rc: int) -> int:
    if rc < 0:
        raise IqError(rc, lib().iq_last_error().decode())
    return rc


def ptr(a) -> int | None:
    """Address of a numpy array (host) or torch tensor (data_ptr)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


class Matrix:
    """A quantized matrix resident on the current CUDA device.

    Mirrors the reference's ``QuantizedMatrix`` (src/gguf.rs:159-785):
    ``forward_rows`` takes row-major f32 input rows and returns row-major f32
    output rows; ``leading_rows`` shares storage.
    """

    def __init__(self, dtype: int, data, rows: int, cols: int, *, _handle=None):
        self.dtype, self.rows, self.cols = dtype, rows, cols
        if _handle is not None:
            self._h = _handle
            return
        h = P()
        if isinstance(data, np.ndarray):
            data = np.ascontiguousarray(data)
            loc = 0
        else:
            loc = 1 if data.is_cuda else 0
            data = data.contiguous()
        self._keep = data
        check(lib().iq_matrix_create(dtype, ptr(data), rows, cols, loc, ctypes.byref(h)))
        self._h = h

    def leading_rows(self, rows: int) -> "Matrix":
        h = P()
        check(lib().iq_matrix_leading_rows(self._h, rows, ctypes.byref(h)))
        return Matrix(self.dtype, None, rows, self.cols, _handle=h)

    def forward_rows(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.cols)
        y = np.empty((x.shape[0], self.rows), np.float32)
        check(lib().iq_matrix_forward_rows(self._h, ptr(x), x.shape[0], ptr(y)))
        return y

    def forward_wide(self, x, stream=None):
        """Many input rows on the tensor cores (Q8_0): ``x`` a CUDA f32 tensor
        [n, cols]; returns a CUDA f32 tensor [n, rows] (enqueued on the
        current stream unless ``stream`` is given)."""
        import torch
        x = x.float().contiguous().view(-1, self.cols)
        y = torch.empty(x.shape[0], self.rows, device=x.device, dtype=torch.float32)
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        check(lib().iq_matrix_forward_wide(self._h, ptr(x), x.shape[0], ptr(y), st))
        return y

    def dequantize(self, ids=None) -> np.ndarray:
        if ids is None:
            out = np.empty((self.rows, self.cols), np.float32)
            check(lib().iq_matrix_dequantize(self._h, None, 0, ptr(out)))
        else:
            ids = np.ascontiguousarray(ids, dtype=np.int32)
            out = np.empty((len(ids), self.cols), np.float32)
            check(lib().iq_matrix_dequantize(self._h, ptr(ids), len(ids), ptr(out)))
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and _lib is not None:
            _lib.iq_matrix_destroy(h)
            self._h = None


def status(stream=None) -> None:
    """Synchronize ``stream`` and raise IqError(IQ_ETIMEDOUT) if a matrix
    product on this device gave up a bounded wait since the last check."""
    check(lib().iq_matrix_status(stream))


def ksplit(dtype: int, rows: int, cols: int) -> int:
    return check(lib().iq_qgemv_ksplit(dtype, rows, cols))
