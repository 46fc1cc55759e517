"""Loader for the C-ABI library ``libhive_b200.so`` (declared in include/hive_b200.h).

The library is built in-tree by :func:`build` (nvcc, sm_100a only).  Loading
fails loudly when it is missing: there is no CPU or Python fallback on the
product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libhive_b200.so")
CSRC = os.path.join(PKG_DIR, "csrc")
SOURCES = ["hv_kernels.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
]

HV_OK = 0


class HiveB200Error(RuntimeError):
    """A C-ABI entry point returned a non-zero hv_status."""


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build(verbose: bool = False) -> str:
    """Compile every CUDA source of the package into libhive_b200.so."""
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", LIB_PATH, *srcs]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=PKG_DIR)
    return LIB_PATH


_vp = C.c_void_p
_i64 = C.c_int64
_int = C.c_int

class HvTree(C.Structure):
    """hv_tree of include/hive_b200.h: the 12 tree arrays + max_nodes."""
    _fields_ = [(n, C.c_void_p) for n in (
        "visit_count", "total_value", "prior", "parent_idx", "virtual_q_penalty", "move_bytes",
        "action_idx", "first_child", "num_children", "is_terminal", "terminal_value", "node_count")] + [
        ("max_nodes", C.c_int32)]


_tp = C.POINTER(HvTree)
_f = C.c_float

_SIGNATURES = {
    "hv_mcts_select": ([_tp, _int, _vp, _vp, _vp, _vp, _vp, _int, _int, _f, _int, _int, _int, _f, _f,
                        _vp, _vp, _vp, _vp, _vp, _vp], _int),
    "hv_mcts_replay": ([_vp, _vp, _vp, _vp, _vp, _int, _int, _vp], _int),
    "hv_mcts_expand": ([_tp, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f,
                        _int, _int, _vp], _int),
    "hv_mcts_expand_slots": ([_tp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _f,
                              _int, _int, _vp], _int),
    "hv_mcts_backprop": ([_tp, _vp, _vp, _vp, _vp, _vp, _int, _int, _vp], _int),
    "hv_mcts_root_noise": ([_tp, _vp, _vp, _int, _f, _f, _int, _vp], _int),
    "hv_mcts_extract_policy": ([_tp, _vp, _vp, _vp, _f, _int, _f, _int, _vp], _int),
    "hv_version": ([], _int),
    "hv_status_string": ([_int], C.c_char_p),
    "hv_get_error": ([_vp, _int], _int),
    "hv_set_wait_limit_ns": ([C.c_uint64], _int),
    "hv_create_initial_states": ([_vp, _i64, _int, _vp], _int),
    "hv_generate_legal_moves": ([_vp, _i64, _vp, _vp, _vp], _int),
    "hv_generate_legal_moves_and_fnn_features": ([_vp, _i64, _vp, _vp, _vp, _vp], _int),
    "hv_extract_fnn_features": ([_vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_stage_host_states": ([_vp, _i64, _vp, _vp], _int),
    "hv_download_moves": ([_vp, _vp, _i64, _vp, _int, _vp], _int),
    "hv_generate_legal_moves_linked": ([_vp, _i64, _vp, _vp, _vp, _vp], _int),
    "hv_fnn_features_linked": ([_vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_fnn_successor_features": ([_vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_fnn_eval_leaves": ([_vp, _vp, _vp, _vp, _i64, _vp, _int, _int, _int, _vp, _vp, _vp, _vp, _vp], _int),
    "hv_fnn_weights_size": ([_int, _int, _int], _int),
    "hv_queen_escape_flags": ([_vp, _i64, _vp, _vp], _int),
    "hv_child_probe": ([_vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _vp], _int),
    "hv_hybrid_encode": ([_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp], _int),
    "hv_hybrid_move_features": ([_vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_generate_legal_moves_and_hybrid_root_features": ([_vp, _i64] + [_vp] * 12, _int),
    "hv_hybrid_trunk_sizes": ([_vp, _vp], _int),
    "hv_hybrid_trunk": ([_vp, _vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _vp], _int),
    "hv_hybrid_trunk_packed_workspace_bytes": ([_i64, _vp], _int),
    "hv_hybrid_trunk_packed": ([_vp, _vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _vp, C.c_size_t, _vp], _int),
    "hv_hybrid_head_weights_size": ([_int, _int, _int], _int),
    "hv_hybrid_eval_leaves": ([_vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _int, _int, _int, _vp, _int, _vp, _vp,
                               _vp, _vp, _vp], _int),
    "hv_hybrid_workspace_bytes": ([_i64, _vp], _int),
    "hv_hybrid_evaluate": ([_vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _int, _int, _int, _vp, _int, _vp, _vp,
                            _vp, _vp, _vp, C.c_size_t, _vp], _int),
    "hv_legal_mask": ([_vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_hybrid_evaluate_noalloc": ([_vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _int, _int, _int, _vp, _int,
                                    _vp, _vp, _vp, _vp, _vp], _int),
    "hv_leaf_rows_workspace_bytes": ([_i64, _i64, _int, _vp], _int),
    "hv_fnn_eval_leaves_rows": ([_vp, _vp, _vp, _vp, _i64, _i64, _vp, _int, _int, _int, _vp, _vp, _vp, _vp, _vp,
                                 C.c_size_t, _vp], _int),
    "hv_hybrid_evaluate_rows": ([_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp, _vp, _vp, _int, _int, _int, _vp, _int,
                                 _vp, _vp, _vp, _vp, _vp, C.c_size_t, _vp], _int),
    "hv_root_tactical_probe": ([_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _vp, _vp, _vp, _vp], _int),
    "hv_apply_moves": ([_vp, _vp, _i64, _vp], _int),
    "hv_check_results": ([_vp, _i64, _vp, _vp], _int),
    "hv_compute_centroids": ([_vp, _i64, _vp, _vp], _int),
    "hv_legal_moves_to_actions": ([_vp, _vp, _vp, _i64, _vp, _vp], _int),
    "hv_generate_positions": ([C.c_uint64, _i64, _i64, _int, _int, _vp, _vp], _int),
}

_lib = None


def exported_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def load() -> C.CDLL:
    """Load libhive_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    lib = C.CDLL(LIB_PATH)
    for name, (args, res) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != HV_OK:
        msg = load().hv_status_string(status).decode()
        raise HiveB200Error(f"{what} failed: hv_status={status} ({msg})")
