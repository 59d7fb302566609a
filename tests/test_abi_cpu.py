"""libq8lin.so builds, loads and exports the whole C ABI; argument errors (no GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "q8lin.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q8lin_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from talechime_b200 import _lib, build

    build.build()
    return _lib.lib()


def test_header_declares_expected_surface():
    fns = header_functions()
    for name in ("q8lin_weight_create", "q8lin_forward", "q8lin_weight_destroy", "q8lin_last_error"):
        assert name in fns


def test_library_exports_every_header_symbol(lib):
    from talechime_b200 import _lib

    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in q8lin.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version(lib):
    assert lib.q8lin_version() == 1


def test_status_strings(lib):
    assert lib.q8lin_status_string(0) == b"Q8LIN_OK"
    assert lib.q8lin_status_string(2) == b"Q8LIN_ERR_SHAPE"
    assert lib.q8lin_status_string(99) == b"Q8LIN_ERR_UNKNOWN"


def test_create_rejects_bad_arguments_before_touching_cuda(lib):
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 68)()
    assert lib.q8lin_weight_create(None, 2, 32, 0, None, ctypes.byref(h)) == 1
    assert lib.q8lin_weight_create(buf, 2, 33, 0, None, ctypes.byref(h)) == 2
    assert b"multiple of the Q8_0 block size" in lib.q8lin_last_error()
    assert lib.q8lin_weight_create(buf, 0, 32, 0, None, ctypes.byref(h)) == 2
    assert lib.q8lin_weight_create(buf, -1, 32, 0, None, ctypes.byref(h)) == 2
    assert lib.q8lin_weight_create(buf, 2, 32, 0, None, None) == 1
    assert h.value is None


def test_forward_rejects_null_handle(lib):
    assert lib.q8lin_forward(None, None, None, 1, None) == 1
    assert b"null" in lib.q8lin_last_error()
    assert lib.q8lin_workspace_size(None, 100) == 0


def test_quantize_rows_shape_checks(lib):
    assert lib.q8lin_quantize_rows(None, 1, 48, None, None, None) == 2
    assert lib.q8lin_quantize_rows(None, 0, 64, None, None, None) == 0
    assert lib.q8lin_quantize_rows(None, 2, 64, None, None, None) == 1


def test_destroy_null_is_noop(lib):
    assert lib.q8lin_weight_destroy(None) == 0


def test_python_surface_rejects_cpu_device():
    import numpy as np

    from talechime_b200 import QMatMul

    with pytest.raises(ValueError):
        QMatMul.from_gguf_blocks(np.zeros(34, np.uint8), 1, 32, device="cpu")
