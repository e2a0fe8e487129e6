"""The C ABI boundary without a GPU: librmoe.so loads, exports exactly what include/rmoe.h
declares, and argument checks fail with a status instead of crashing."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "rmoe.h")).read()
    return sorted(set(re.findall(r"RMOE_API\s+[\w\s\*]*?\b(rmoe_\w+)\s*\(", src)))


def test_header_declares_the_hot_path_entry_points():
    syms = declared_symbols()
    for name in ("rmoe_route", "rmoe_dispatch", "rmoe_moe_forward", "rmoe_moe_forward_host",
                 "rmoe_matmul_mxfp4", "rmoe_matmul_i4_grouped", "rmoe_matmul_f32",
                 "rmoe_upload_expert", "rmoe_layer_create"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from rabbit_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    # and the Python binding covers every declared entry point
    assert set(declared_symbols()) == set(_lib.PROTOTYPES)


def test_abi_version_and_status_strings():
    from rabbit_b200 import _lib

    lib = _lib.load()
    assert lib.rmoe_abi_version() == 4
    assert lib.rmoe_status_string(2) == b"shape mismatch"


def test_null_arguments_fail_with_invalid_arg():
    from rabbit_b200 import _lib

    lib = _lib.load()
    assert lib.rmoe_init(0, None) == 1
    assert b"null" in lib.rmoe_last_error()
    assert lib.rmoe_layer_create(None, None, None) == 1
    assert lib.rmoe_upload_router(None, None, 0, 0) == 1
    assert lib.rmoe_route(None, None, 0, 1, None, None, None) == 1
    assert lib.rmoe_moe_forward(None, None, 0, 1, None, None, None, None) == 1
    assert lib.rmoe_matmul_mxfp4(None, None, 0, None, None, 1, 32, 1, None) == 1


def test_missing_library_fails_loudly(tmp_path):
    from rabbit_b200 import _lib

    saved = _lib._lib
    _lib._lib = None
    try:
        with pytest.raises(ImportError, match="no CPU fallback"):
            _lib.load(str(tmp_path / "librmoe.so"))
    finally:
        _lib._lib = saved
