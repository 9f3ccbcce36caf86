"""CPU tests of the C-ABI boundary: the library builds for sm_100a, loads
without a GPU, exports every symbol include/rta.h declares, and rejects bad
arguments with a status code (host-side validation, no device work)."""
import ctypes

from rta_b200 import _lib


def test_library_builds_and_exports_header_symbols():
    lib = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib._SIGNATURES) <= set(names)
    assert lib.rta_version().decode().endswith("sm_100a")


def test_argument_validation_without_device():
    lib = _lib.load()
    assert lib.rta_gemv(12, None, 16, 256, None, 1, None, 0, None) == _lib.RTA_E_ARG
    assert b"rta_gemv" in lib.rta_last_error()
    assert lib.rta_quantize(3, None, 1, None, None) == _lib.RTA_E_ARG
    assert lib.rta_readout(14, None, 16, 256, None, 9, None, None, None, None, None) == _lib.RTA_E_ARG
    word = ctypes.c_uint32(0)
    assert lib.rta_workspace_error(None, 0, None, ctypes.byref(word)) == _lib.RTA_E_ARG
    assert lib.rta_attention_workspace_bytes(16, 4, 256, 8) > 16 * 8 * 256 * 4

