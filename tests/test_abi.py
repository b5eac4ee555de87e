"""libiq loads and exports every symbol include/iq.h declares (no GPU work)."""
import ctypes

from inferq_b200 import _lib


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    names = _lib.declared_symbols()
    assert "iq_matrix_forward_rows" in names and "iq_last_error" in names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_errors_are_reported_not_raised():
    L = _lib.lib()
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 64)()
    rc = L.iq_matrix_create(3, buf, 1, 32, 0, ctypes.byref(h))  # Q4_1: unsupported
    assert rc == -4
    assert b"unsupported" in L.iq_last_error()
    assert L.iq_qgemv_ksplit(12, 2048, 100) == -1  # not a whole block


def test_ksplit_depends_only_on_shape():
    assert _lib.ksplit(12, 248320, 2048) == 1
    assert _lib.ksplit(8, 2048, 4096) == 8
    assert _lib.ksplit(14, 2048, 512) == 2
