"""The C-ABI library loads, exports every declared symbol and validates arguments (CPU only).

No test here launches a kernel: the argument checks run before any CUDA call.
"""

from __future__ import annotations

import ctypes as C
import glob
import os
import re

import pytest

from actfold_b200 import _lib
import actfold_b200.kernels  # noqa: F401  (registers GEMM/attention signatures)
import actfold_b200.llada  # noqa: F401  (registers the folded-pass signatures)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(af_[a-z0-9_]+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from actfold_b200.build import build

        build()
    return _lib.load()


def test_header_declares_functions():
    names = _declared_functions()
    assert {"af_gate", "af_merge_rows", "af_gather_rows_masked", "af_version", "af_last_error_string"} <= names


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(_declared_functions()):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_string(lib):
    assert lib.af_version().decode().startswith("actfold_b200")


def test_gate_rejects_null_pointers(lib):
    st = lib.af_gate(None, 0, 0, None, 0, 0, 1, 1, 8, 2, 0, 0.95, 1e-8, 1.0, None, 1, None, None, None, 1, None, None)
    assert st == _lib.AF_ERR_ARG
    assert "null" in lib.af_last_error_string().decode()


def test_gate_rejects_bad_dtype_and_shape(lib):
    buf = C.create_string_buffer(64)
    p = C.cast(buf, C.c_void_p).value
    assert lib.af_gate(p, 0, 0, p, 0, 0, 1, 1, 8, 7, 0, 0.95, 1e-8, 1.0, p, 1, None, None, None, 1, None, None) == _lib.AF_ERR_ARG
    assert lib.af_gate(p, 0, 0, p, 0, 0, 1, 1, 0, 2, 0, 0.95, 1e-8, 1.0, p, 1, None, None, None, 1, None, None) == _lib.AF_ERR_ARG
    # compaction outputs need a count buffer
    assert lib.af_gate(p, 0, 0, p, 0, 0, 1, 1, 8, 2, 0, 0.95, 1e-8, 1.0, p, 1, None, None, p, 1, None, None) == _lib.AF_ERR_ARG


def test_row_kernels_reject_null_and_mode(lib):
    assert lib.af_merge_rows(None, 0, 0, None, 0, 0, None, 0, None, 0, 0, 1, 1, 16, None) == _lib.AF_ERR_ARG
    buf = C.create_string_buffer(64)
    p = C.cast(buf, C.c_void_p).value
    assert lib.af_gather_rows_masked(p, 0, 0, p, 0, None, 3, p, 0, 0, 1, 1, 16, None) == _lib.AF_ERR_ARG
    assert lib.af_gather_rows_index(None, 0, 0, None, 1, 1, None, 0, 0, 16, None) == _lib.AF_ERR_ARG


def test_check_maps_status_to_exceptions(lib):
    lib.af_merge_rows(None, 0, 0, None, 0, 0, None, 0, None, 0, 0, 1, 1, 16, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.AF_ERR_ARG)
    with pytest.raises(TimeoutError):
        _lib.check(_lib.AF_ERR_TIMEOUT)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.AF_ERR_CUDA)
