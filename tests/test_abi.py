"""The C-ABI library loads without a GPU and exports every declared symbol."""

import ctypes
import re

from .conftest import ROOT

HEADER = ROOT / "include" / "matrixman_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*int\s+(mm_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 60
    assert "mm_conv2d" in names and "mm_alloc" in names and "mm_yolo_decode" in names


def test_library_exports_every_declared_symbol():
    from matrixman_b200 import _lib
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/matrixman_b200.h but not exported"


def test_binding_covers_header():
    from matrixman_b200 import _lib
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_abi_version_and_errors_without_gpu():
    from matrixman_b200 import _lib
    lib = _lib.load()
    assert lib.mm_abi_version() == 1
    n = ctypes.c_int(-1)
    lib.mm_device_count(ctypes.byref(n))
    assert n.value >= 0
    # A call on an uninitialised device fails cleanly with a message.
    out = ctypes.c_void_p()
    status = lib.mm_alloc(0, 16, 0, None, ctypes.byref(out))
    assert status == _lib.MM_ERR_STATE
    assert "not initialised" in _lib.last_error()


def test_descriptor_validation_without_gpu():
    from matrixman_b200 import _lib
    lib = _lib.load()
    bad = _lib.make_tensor(0, (2, 3), (3, 1))  # null data with elements
    good = _lib.make_tensor(0, (0,), (1,))
    assert lib.mm_unary(0, ctypes.byref(bad), ctypes.byref(bad), 0.0, 0.0, None) == _lib.MM_ERR_INVALID
    # Empty tensors are a no-op.
    assert lib.mm_unary(0, ctypes.byref(good), ctypes.byref(good), 0.0, 0.0, None) == _lib.MM_OK
    neg = _lib.make_tensor(8, (2,), (-1,))
    assert lib.mm_fill(ctypes.byref(neg), 0.0, None) == _lib.MM_ERR_INVALID


def test_hooks_extension_source_present():
    assert (ROOT / "matrixman_b200" / "csrc" / "privateuse1_hooks.cpp").exists()
