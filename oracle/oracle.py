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


def reference_dir() -> str:
    """Root of the reference source tree (chrismejias/hive_neuralnet): the
    ``HIVE_REFERENCE`` environment variable, else a directory named
    ``reference`` beside this repository.  Only fixture generators and the
    reference build of the oracle read it; GPU tests and the bench never do."""
    env = os.environ.get("HIVE_REFERENCE")
    if env:
        return os.path.abspath(env)
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def reference_available() -> bool:
    return os.path.isdir(os.path.join(reference_dir(), "hive_gpu", "csrc"))


def build(ref: bool = True) -> None:
    """Compile liboracle.so (and the reference build when the tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref and reference_available():
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"HIVE_REFERENCE={reference_dir()}"], check=True)


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
        self._hyb = sig("hybrid_encode_batch", [_u8p, _u8p, _i32p, _i64, _f32p, _i32p, _i32p, _i32p, _u8p,
                                                _f32p, _i32p, _f32p, _int])
        self._mask = sig("legal_mask_batch", [_u8p, _u8p, _i32p, _i64, _f32p])
        self._tac = sig("tactical_probe_batch", [_u8p, _u8p, _i32p, _f32p, _i64, _int, _int, _int,
                                                 _i64p, _u8p, _u8p, _int])
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


    def legal_mask(self, states, moves, num_legal):
        """legal_mask_kernel outputs [B, 85834] f32 (reference build only)."""
        states = np.ascontiguousarray(states, np.uint8)
        out = np.zeros((states.shape[0], 85834), np.float32)
        self._mask(states, np.ascontiguousarray(moves, np.uint8), np.ascontiguousarray(num_legal, np.int32),
                   states.shape[0], out)
        return out

    def tactical_probe(self, states, moves, num_legal, priors, w1=True, chk=True, w2=True, threads: int = 0):
        """root_tactical_probe_batch: (winning [B] i64, allowed [B,256] u8, forced [B] u8)."""
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        win = np.zeros(b, np.int64)
        allowed = np.zeros((b, MAX_MOVES), np.uint8)
        forced = np.zeros(b, np.uint8)
        self._tac(states, np.ascontiguousarray(moves, np.uint8), np.ascontiguousarray(num_legal, np.int32),
                  np.ascontiguousarray(priors, np.float32), b, int(w1), int(chk), int(w2), win, allowed,
                  forced, threads)
        return win, allowed, forced


    def hybrid_encode(self, states, moves, num_legal, threads: int = 0):
        """hybrid_transformer_encode_with_moves_batch + hybrid_transformer_move_features_batch outputs:
        (token_features [B,28,27], q, r, z [B,28] i32, mask [B,28] u8, global [B,6], num_tokens [B],
        move_features [B,256,31])."""
        states = np.ascontiguousarray(states, np.uint8)
        b = states.shape[0]
        tf = np.zeros((b, 28, 27), np.float32)
        tq, tr, tz = (np.zeros((b, 28), np.int32) for _ in range(3))
        tm = np.zeros((b, 28), np.uint8)
        gf = np.zeros((b, 6), np.float32)
        nt = np.zeros(b, np.int32)
        mf = np.zeros((b, MAX_MOVES, 31), np.float32)
        self._hyb(states, np.ascontiguousarray(moves, np.uint8), np.ascontiguousarray(num_legal, np.int32), b,
                  tf, tq, tr, tz, tm, gf, nt, mf, threads)
        return tf, tq, tr, tz, tm, gf, nt, mf


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


# ---------------------------------------------------------------------------
# MCTS tree arrays and the sequential tree operations (orc_mcts_* / ref_mcts_*)
# ---------------------------------------------------------------------------
class _TreePtrs(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("vc", "tv", "pr", "pa", "vq", "mb", "ai", "fc", "nc", "it",
                                          "tval", "cnt")] + [("max_nodes", C.c_int32)]


TREE_FIELDS = (("visit_count", np.int32, 0), ("total_value", np.float32, 0), ("prior", np.float32, 0),
               ("parent_idx", np.int32, -1), ("virtual_q_penalty", np.float32, 0),
               ("move_bytes", np.uint8, 0), ("action_idx", np.int32, -1), ("first_child", np.int32, -1),
               ("num_children", np.int32, 0), ("is_terminal", np.int8, 0), ("terminal_value", np.float32, 0),
               ("node_count", np.int32, 1))


class TreeArrays:
    """numpy copy of the reference's SoA tree (binding order of bindings.cpp:130-135)."""

    def __init__(self, B: int, max_nodes: int):
        self.B, self.max_nodes = B, max_nodes
        for name, dt, fill in TREE_FIELDS:
            shape = (B,) if name == "node_count" else ((B, max_nodes, 6) if name == "move_bytes" else (B, max_nodes))
            setattr(self, name, np.full(shape, fill, dtype=dt))
        self.child_init_q = np.zeros((B, max_nodes), np.float32)

    def copy(self) -> "TreeArrays":
        t = TreeArrays.__new__(TreeArrays)
        t.B, t.max_nodes = self.B, self.max_nodes
        for name, _, _ in TREE_FIELDS:
            setattr(t, name, getattr(self, name).copy())
        t.child_init_q = self.child_init_q.copy()
        return t

    def arrays(self):
        return [getattr(self, n) for n, _, _ in TREE_FIELDS]

    def ptrs(self) -> _TreePtrs:
        a = self.arrays()
        return _TreePtrs(*[x.ctypes.data for x in a], self.max_nodes)

    def equal(self, other: "TreeArrays") -> list[str]:
        bad = []
        for name, _, _ in TREE_FIELDS + (("child_init_q", None, None),):
            x, y = getattr(self, name), getattr(other, name)
            if x.dtype == np.float32:
                x, y = x.view(np.uint32), y.view(np.uint32)
            if not np.array_equal(x, y):
                bad.append(name)
        return bad


def _p(a):
    return None if a is None else np.ascontiguousarray(a).ctypes.data


def mcts_select(lib_name: str, tree: TreeArrays, mode: int, game_active, root_nodes, alive_mask=None,
                root_slots=None, num_candidates=1, max_root_children=256, c_puct=1.25, W=1, det=False,
                sigma=4.0, q_penalty=0.0):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    fn = getattr(lib, f"{lib_name}_mcts_select")
    B = tree.B
    total = W * num_candidates * B if mode == 2 else W * B
    leaf = np.zeros(total, np.int32)
    paths = np.zeros((total, 128, 6), np.uint8)
    plen = np.zeros(total, np.int32)
    vlp = np.zeros((total, 128), np.int32)
    vll = np.zeros(total, np.int32)
    ptrs = tree.ptrs()
    fn(C.byref(ptrs), C.c_int(mode), C.c_void_p(tree.child_init_q.ctypes.data),
       C.c_void_p(_p(game_active)), C.c_void_p(_p(root_nodes)), C.c_void_p(_p(alive_mask)),
       C.c_void_p(_p(root_slots)), C.c_int(num_candidates), C.c_int(max_root_children),
       C.c_float(c_puct), C.c_int(B), C.c_int(W), C.c_int(int(det)), C.c_float(sigma), C.c_float(q_penalty),
       C.c_void_p(leaf.ctypes.data), C.c_void_p(paths.ctypes.data), C.c_void_p(plen.ctypes.data),
       C.c_void_p(vlp.ctypes.data), C.c_void_p(vll.ctypes.data))
    return leaf, paths, plen, vlp, vll


def mcts_replay(lib_name: str, root_states, paths, plen, leaf, B):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    total = len(leaf)
    out = np.zeros((total, STATE_BYTES), np.uint8)
    rs = np.ascontiguousarray(root_states)
    getattr(lib, f"{lib_name}_mcts_replay")(C.c_void_p(rs.ctypes.data), C.c_void_p(out.ctypes.data),
                                            C.c_void_p(paths.ctypes.data), C.c_void_p(plen.ctypes.data),
                                            C.c_void_p(leaf.ctypes.data), C.c_int(B), C.c_int(total))
    return out


def mcts_expand_dense(lib_name: str, tree: TreeArrays, child_q, leaf, leaf_states, legal, num_legal,
                      priors, results, values=None, vl_paths=None, vl_len=None, q_penalty=0.0,
                      with_backprop=True):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    total = len(leaf)
    was = np.zeros(total, np.int8)
    keep = [np.ascontiguousarray(x) for x in (child_q, leaf, leaf_states, legal, num_legal, priors, results)]
    vals = np.ascontiguousarray(values if values is not None else np.zeros(total, np.float32))
    vlp = np.ascontiguousarray(vl_paths if vl_paths is not None else np.zeros((total, 128), np.int32))
    vll = np.ascontiguousarray(vl_len if vl_len is not None else np.zeros(total, np.int32))
    ptrs = tree.ptrs()
    getattr(lib, f"{lib_name}_mcts_expand_dense")(
        C.byref(ptrs), C.c_void_p(tree.child_init_q.ctypes.data), *[C.c_void_p(k.ctypes.data) for k in keep],
        C.c_void_p(vals.ctypes.data), C.c_void_p(vlp.ctypes.data), C.c_void_p(vll.ctypes.data),
        C.c_int(tree.B), C.c_int(total), C.c_float(q_penalty), C.c_int(int(with_backprop)),
        C.c_void_p(was.ctypes.data))
    return was


def mcts_expand_action(lib_name: str, tree: TreeArrays, mode: int, leaf, leaf_states, legal, num_legal,
                       probs, results, values=None, vl_paths=None, vl_len=None, was_expanded=None):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    total = len(leaf)
    was = np.ascontiguousarray(was_expanded if was_expanded is not None else np.zeros(total, np.int8))
    keep = [np.ascontiguousarray(x) for x in (leaf, leaf_states, legal, num_legal, probs, results)]
    vals = np.ascontiguousarray(values if values is not None else np.zeros(total, np.float32))
    vlp = np.ascontiguousarray(vl_paths if vl_paths is not None else np.zeros((total, 128), np.int32))
    vll = np.ascontiguousarray(vl_len if vl_len is not None else np.zeros(total, np.int32))
    ptrs = tree.ptrs()
    getattr(lib, f"{lib_name}_mcts_expand_action")(
        C.byref(ptrs), *[C.c_void_p(k.ctypes.data) for k in keep], C.c_void_p(vals.ctypes.data),
        C.c_void_p(vlp.ctypes.data), C.c_void_p(vll.ctypes.data), C.c_int(tree.B), C.c_int(total),
        C.c_int(mode), C.c_void_p(was.ctypes.data))
    return was


def mcts_extract_policy(lib_name: str, tree: TreeArrays, move_numbers, root_nodes, temperature,
                        temp_drop_move, pruning_threshold):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    pol = np.zeros((tree.B, 85834), np.float32)
    mn = np.ascontiguousarray(move_numbers, np.int32)
    rn = np.ascontiguousarray(root_nodes, np.int32)
    ptrs = tree.ptrs()
    getattr(lib, f"{lib_name}_mcts_extract_policy")(
        C.byref(ptrs), C.c_void_p(pol.ctypes.data), C.c_void_p(mn.ctypes.data), C.c_void_p(rn.ctypes.data),
        C.c_float(temperature), C.c_int(temp_drop_move), C.c_float(pruning_threshold), C.c_int(tree.B))
    return pol


def mcts_root_noise(lib_name: str, tree: TreeArrays, noise, root_nodes, dir_eps, root_policy_temp):
    lib = (oracle() if lib_name == "orc" else ref()).lib
    nz = np.ascontiguousarray(noise, np.float32)
    rn = np.ascontiguousarray(root_nodes, np.int32)
    ptrs = tree.ptrs()
    getattr(lib, f"{lib_name}_mcts_root_noise")(
        C.byref(ptrs), C.c_void_p(nz.ctypes.data), C.c_void_p(rn.ctypes.data), C.c_int(nz.shape[1]),
        C.c_float(dir_eps), C.c_float(root_policy_temp), C.c_int(tree.B))
