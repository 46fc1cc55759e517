"""ctypes bindings for the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two libraries share one calling convention:

* ``liboracle.so`` -- the plain-C restatement in ``oracle/hive_oracle.c``;
* ``_ref/libhive_ref.so`` -- the reference's own game-logic headers compiled
  on the host by ``oracle/ref_driver.cpp`` (present only where the reference
  tree was available at build time).

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use this
module, as the checker and the timed CPU baseline.  The product path
(``hive_neuralnet_b200``) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
STATE_BYTES = 3424
MOVE_BYTES = 6
MAX_MOVES = 256
FEAT = 122
WORDS = 9

_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i64 = C.c_int64
_int = C.c_int


def build(ref: bool = True) -> None:
    """Compile liboracle.so (and the reference build when the tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref and os.path.isdir("/root/reference/hive_gpu/csrc"):
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.path = path
        self.lib = C.CDLL(path)
        p = prefix
        L = self.lib

        def sig(name, args, res=None):
            f = getattr(L, p + name, None)
            if f is None:
                return None
            f.argtypes = args
            f.restype = res
            return f

        self._lmf = sig("legal_moves_features_batch", [_u8p, _i64, _u8p, _i32p, _f32p, _int])
        self._feat = sig("features_batch", [_u8p, _u8p, _i32p, _i64, _f32p, _int])
        self._compact = sig("compact_moves_batch", [_u8p, _i64, _u8p, _i32p, _int])
        self._succ = sig("successor_features_batch", [_u8p, _u8p, _i64p, _i64p, _i64, _f32p, _int])
        self._apply = sig("apply_moves_batch", [_u8p, _u8p, _i64])
        self._ap = sig("articulation_batch", [_u8p, _i64, _u64p, _int])
        self._act = sig("actions_batch", [_u8p, _u8p, _i32p, _i64, _i32p, _i32p])
        self._qe = sig("queen_escape_batch", [_u8p, _i64, _u8p])
        self._gen = sig("generate_positions",
                        [C.c_uint64, _i64, _i64, _int, _int, _u8p, _int])

    # -- batched helpers returning numpy arrays ---------------------------
    def generate_positions(self, seed: int, first_game: int, count: int, max_ply: int,
                           expansion_mask: int, threads: int = 0) -> np.ndarray:
        out = np.zeros((count, STATE_BYTES), np.uint8)
        self._gen(seed, first_game, count, max_ply, expansion_mask, out, threads)
        return out

    def legal_moves_features(self, states: np.ndarray, threads: int = 0):
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        moves = np.zeros((b, MAX_MOVES, MOVE_BYTES), np.uint8)
        nl = np.zeros(b, np.int32)
        feats = np.zeros((b, FEAT), np.float32)
        self._lmf(states, b, moves, nl, feats, threads)
        return moves, nl, feats

    def features(self, states, moves, num_legal, threads: int = 0):
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        feats = np.zeros((b, FEAT), np.float32)
        self._feat(states, np.ascontiguousarray(moves, np.uint8),
                   np.ascontiguousarray(num_legal, np.int32), b, feats, threads)
        return feats

    def compact_moves(self, states, threads: int = 0):
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        moves = np.zeros((b, MAX_MOVES, MOVE_BYTES), np.uint8)
        nl = np.zeros(b, np.int32)
        self._compact(states, b, moves, nl, threads)
        return moves, nl

    def successor_features(self, states, moves, action_to_root, move_indices, threads: int = 0):
        n = int(len(action_to_root))
        feats = np.zeros((n, FEAT), np.float32)
        self._succ(np.ascontiguousarray(states, np.uint8), np.ascontiguousarray(moves, np.uint8),
                   np.ascontiguousarray(action_to_root, np.int64),
                   np.ascontiguousarray(move_indices, np.int64), n, feats, threads)
        return feats

    def apply_moves(self, states, moves):
        out = np.array(states, dtype=np.uint8, copy=True, order="C")
        self._apply(out, np.ascontiguousarray(moves, np.uint8), out.shape[0])
        return out

    def articulation(self, states, threads: int = 0):
        states = np.ascontiguousarray(states, np.uint8)
        out = np.zeros((states.shape[0], WORDS), np.uint64)
        self._ap(states, states.shape[0], out, threads)
        return out

    def actions(self, states, moves, num_legal):
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        act = np.zeros((b, MAX_MOVES), np.int32)
        cen = np.zeros((b, 2), np.int32)
        self._act(states, np.ascontiguousarray(moves, np.uint8),
                  np.ascontiguousarray(num_legal, np.int32), b, act, cen)
        return act, cen

    def queen_escape(self, states):
        states = np.ascontiguousarray(states, np.uint8)
        out = np.zeros(states.shape[0], np.uint8)
        self._qe(states, states.shape[0], out)
        return out


_oracle = None
_ref = None


def oracle() -> _Lib:
    """The C restatement (always available once built)."""
    global _oracle
    if _oracle is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build(ref=False)
        _oracle = _Lib(path, "orc_")
    return _oracle


def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libhive_ref.so"))


def ref() -> _Lib:
    """The reference's own headers compiled on the host (None if not built)."""
    global _ref
    if _ref is None:
        if not ref_available():
            return None
        _ref = _Lib(os.path.join(HERE, "_ref", "libhive_ref.so"), "ref_")
    return _ref
