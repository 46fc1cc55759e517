"""CPU tests of the C-ABI boundary: the library loads and exports every
symbol that include/hive_b200.h declares (no compute calls without a GPU)."""
import ctypes
import os
import re

import pytest

from hive_neuralnet_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hive_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        _lib.build()
    return _lib.load()


def test_header_declares_bound_symbols():
    assert _declared() == _lib.exported_symbols()


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings(lib):
    assert lib.hv_version() == 1
    assert lib.hv_status_string(0) == b"ok"
    assert b"invalid" in lib.hv_status_string(1)


def test_invalid_arguments_rejected_without_gpu(lib):
    # argument validation happens before any CUDA call
    assert lib.hv_generate_legal_moves(None, 4, None, None, None) == 1
    assert lib.hv_generate_legal_moves(None, -1, None, None, None) == 1
    misaligned = ctypes.c_void_p(8)
    assert lib.hv_generate_legal_moves_and_fnn_features(misaligned, 1, None, None, None, None) == 1
    # the fused entry keeps 8-byte working data in its feature rows
    aligned = ctypes.c_void_p(256)
    assert lib.hv_generate_legal_moves_and_fnn_features(aligned, 1, aligned, aligned, ctypes.c_void_p(260),
                                                        None) == 1
    assert lib.hv_apply_moves(None, None, 0, None) == 0  # empty batch is a no-op


def test_loader_fails_loudly_without_library(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _lib.load()
