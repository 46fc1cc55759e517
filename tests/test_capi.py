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


def test_download_and_packed_trunk_arguments_without_gpu(lib):
    v = ctypes.c_void_p(256)
    # the row prefix is a multiple of 8 moves in 0..256; counts are not negative
    for bad in (-8, 12, 264):
        assert lib.hv_download_moves(v, v, 4, v, bad, None) == 1
    assert lib.hv_download_moves(v, v, -1, v, 64, None) == 1
    assert lib.hv_download_moves(None, v, 4, v, 64, None) == 1
    assert lib.hv_download_moves(None, None, 0, None, 64, None) == 0  # empty chunk: nothing to do
    # the packed trunk's slot table: two counters and one entry per position
    need = ctypes.c_size_t(0)
    assert lib.hv_hybrid_trunk_packed_workspace_bytes(1000, ctypes.addressof(need)) == 0
    assert need.value == 16 + 8 * 1000
    assert lib.hv_hybrid_trunk_packed_workspace_bytes(-1, ctypes.addressof(need)) == 1
    # workspace missing, off a 16-byte boundary or too small
    args = [v] * 5 + [1000, 27, v, v, v]
    assert lib.hv_hybrid_trunk_packed(*args, None, 16 + 8 * 1000, None) == 1
    assert lib.hv_hybrid_trunk_packed(*args, ctypes.c_void_p(264), 16 + 8 * 1000, None) == 1
    assert lib.hv_hybrid_trunk_packed(*args, v, 8 * 1000, None) == 1


def test_host_pipeline_rejects_bad_prefix_without_gpu():
    import torch
    from hive_neuralnet_b200.hive_gpu import load_extension
    ext = load_extension()
    st = torch.zeros((4, 3424), dtype=torch.uint8)
    for bad in (-8, 12, 264):
        with pytest.raises(ValueError):
            ext.generate_legal_moves_and_fnn_features_host(st, 4, move_prefix=bad)


def test_loader_fails_loudly_without_library(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError):
        _lib.load()
