"""The C-ABI library loads and exports every symbol the public headers declare."""
import ctypes as C
import os
import re

import pytest

from diskmule_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fn)).read()
        names.update(re.findall(r"DM_API[^;(]*?\b(dm_\w+)\s*\(", text, flags=re.S))
    return sorted(names)


def test_headers_declare_the_boundary():
    names = declared_symbols()
    assert "dm_moe_forward" in names and "dm_cuda_matvec" in names
    assert len(names) >= 25


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_declared_symbol(name):
    lib = C.CDLL(N.LIB_PATH)
    assert hasattr(lib, name), name


def test_python_signatures_cover_every_declared_symbol():
    assert set(declared_symbols()) <= set(N.SIGNATURES)


def test_status_strings_and_no_device_error():
    L = N.lib()
    assert L.dm_status_string(N.OK) == b"ok"
    assert b"expert" in L.dm_status_string(N.ERR_INVALID_EXPERT)
    h = C.c_void_p()
    rc = L.dm_cuda_create(0, C.byref(h))
    if rc == N.OK:
        L.dm_cuda_destroy(h)
        pytest.skip("a GPU is visible")
    assert rc == N.ERR_NO_DEVICE
    assert b"device" in L.dm_last_error_message()


def test_null_arguments_are_rejected_before_any_device_work():
    L = N.lib()
    assert L.dm_cuda_create(0, None) == N.ERR_INVALID_ARGUMENT
    assert L.dm_moe_forward(None, None, None, 1, None, None, None) == N.ERR_INVALID_ARGUMENT
    assert L.dm_moe_layer_create(None, None, None) == N.ERR_INVALID_ARGUMENT
