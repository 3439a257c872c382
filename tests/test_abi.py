"""CPU checks of the C ABI: the library loads, exports every entry point the
headers declare, and its pure helpers and error path work without a GPU."""
import ctypes

import pytest

from rustyllm_b200 import _lib


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _lib.declared_symbols()
    assert len(declared) >= 13
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding covers the whole ABI
    assert set(declared) <= set(_lib.SIGNATURES)


def test_version_and_block_sizes():
    L = _lib.lib()
    assert b"sm_100a" in L.rq_version()
    assert L.rq_block_bytes(2) == 18 and L.rq_block_elems(2) == 32
    assert L.rq_block_bytes(12) == 144 and L.rq_block_elems(12) == 256
    assert L.rq_block_bytes(11) == 110 and L.rq_block_elems(11) == 256
    assert L.rq_block_bytes(99) == 0 and L.rq_block_elems(99) == 0


def test_null_arguments_report_errors():
    L = _lib.lib()
    rc = L.rq_init(0, None)
    assert rc == 1
    assert "NULL" in _lib.last_error()
    rc = L.rq_linear(None, None, None, None, 1, None)
    assert rc == 1
    with pytest.raises(_lib.RqError, match="rq_linear"):
        _lib.check(rc)


def test_init_without_usable_device_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = ctypes.c_void_p()
    rc = _lib.lib().rq_init(0, ctypes.byref(h))
    assert rc != 0 and not h.value
    assert _lib.last_error()
