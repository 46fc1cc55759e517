"""Drop-in mirror of the reference's ``hive_gpu.load_extension()`` module.

The reference loads a pybind/torch extension ``hive_gpu_ext``
(hive_gpu/__init__.py:45-89, functions in hive_gpu/csrc/bindings.cpp:254-476).
:func:`load_extension` here returns an object with the same attribute names,
positional/keyword signatures, output dtypes/shapes and constants, backed by
the sm_100a kernels of ``libhive_b200.so`` through its C ABI.  Differences in
behaviour that are deliberate:

* every call validates dtype / device / contiguity / sizes once and raises
  ``ValueError`` instead of reading out of bounds;
* kernels run on ``torch.cuda.current_stream()`` (the reference uses the
  legacy default stream and a few device-wide synchronisations);
* there is no Python or CPU fallback: a missing library raises ImportError.
"""
from __future__ import annotations

import torch

from . import _lib

# constants, bindings.cpp:445-475
BOARD_SIZE = 23
NUM_CELLS = 529
MAX_LEGAL_MOVES = 256
MAX_STACK = 5
SIZEOF_HIVE_STATE = 3424
SIZEOF_GPU_MOVE = 6
OFF_TURN = 3412
OFF_QUEEN_PLACED = 3414
OFF_RESULT = 3415
OFF_STUNNED_CELL = 3416
OFF_QUEEN_CELL = 3392
OFF_HANDS = 3396
MAX_ENC_NODES = 48
MAX_ENC_EDGES = 200
NODE_FEAT_DIM = 25
EDGE_FEAT_DIM = 9
GLOBAL_FEAT_DIM = 6
HYBRID_MAX_NODES = 48
HYBRID_MAX_EDGES = 640
HYBRID_MAX_PIECE_TOKENS = 28
HYBRID_NODE_FEAT_DIM = 27
HYBRID_MOVE_FEAT_DIM = 31
HYBRID_EDGE_FEAT_DIM = 3
HYBRID_GLOBAL_FEAT_DIM = 6
ENC_GRID = 17
ACTION_SPACE_SIZE = 85834
PASS_ACTION_INDEX = 85833
MOVEMENT_OFFSET = 2312
DEFAULT_MAX_TREE_NODES = 65536
MAX_TREE_DEPTH = 128
FNN_FEAT_DIM = 122

_OUT_OF_SCOPE = (
    "encode_states_batch", "hybrid_gnn_encode_batch", "hybrid_gnn_encode_with_moves_batch",
    "compute_mobility_batch", "endgame_hit_mask_batch", "debug_tactical_state_batch",
    "fnn_selfplay_batch", "prs_v2_classify_batch",
)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, rows: int | None = None,
          tail: tuple | None = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise ValueError(f"{name}: expected a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor, got {t.device}")
    if t.dtype != dtype:
        raise ValueError(f"{name}: expected dtype {dtype}, got {t.dtype}")
    if rows is not None and (t.dim() == 0 or t.shape[0] < rows):
        raise ValueError(f"{name}: expected at least {rows} rows, got shape {tuple(t.shape)}")
    if tail is not None:
        flat = t.reshape(t.shape[0], -1) if t.dim() else t
        if flat.shape[1:].numel() != int(torch.Size(tail).numel()):
            raise ValueError(f"{name}: expected trailing shape {tail}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        t = t.contiguous()
    return t


class HiveGPUExtension:
    """Module-like object returned by :func:`load_extension`."""

    def __init__(self):
        self._lib = _lib.load()
        for k, v in globals().items():
            if k.isupper() and isinstance(v, int):
                setattr(self, k, v)

    # -- tables / profiling (bindings.cpp:257-262) ---------------------------
    def initialize_tables(self) -> None:
        """Grid tables are compile-time constants here: nothing to upload, on any device."""

    def reset_movegen_profile(self) -> None:
        """Per-kernel counters come from ncu (profiles/); no device counters to reset."""

    def get_movegen_profile(self) -> torch.Tensor:
        return torch.zeros(27, dtype=torch.int64)

    # -- state ops ------------------------------------------------------------
    def create_initial_states(self, batch_size: int, expansion_mask: int = 0) -> torch.Tensor:
        states = torch.empty((batch_size, SIZEOF_HIVE_STATE), dtype=torch.uint8, device="cuda")
        _lib.check(self._lib.hv_create_initial_states(_ptr(states), batch_size, expansion_mask,
                                                      _stream(states.device)),
                   "create_initial_states")
        return states

    def generate_legal_moves_batch(self, states: torch.Tensor, batch_size: int):
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        moves = torch.empty((batch_size, MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=dev)
        num_legal = torch.empty((batch_size,), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_generate_legal_moves(_ptr(states), batch_size, _ptr(moves),
                                                         _ptr(num_legal), _stream(dev)),
                       "generate_legal_moves_batch")
        return moves, num_legal

    def generate_legal_moves_and_fnn_features_batch(self, states: torch.Tensor, batch_size: int):
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        moves = torch.empty((batch_size, MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=dev)
        num_legal = torch.empty((batch_size,), dtype=torch.int32, device=dev)
        feats = torch.empty((batch_size, FNN_FEAT_DIM), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_generate_legal_moves_and_fnn_features(
                _ptr(states), batch_size, _ptr(moves), _ptr(num_legal), _ptr(feats), _stream(dev)),
                "generate_legal_moves_and_fnn_features_batch")
        return moves, num_legal, feats

    def extract_fnn_features_batch(self, states: torch.Tensor, legal_moves: torch.Tensor,
                                   num_legal: torch.Tensor, batch_size: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, batch_size,
                            (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, batch_size)
        dev = states.device
        feats = torch.empty((batch_size, FNN_FEAT_DIM), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_extract_fnn_features(_ptr(states), _ptr(legal_moves), _ptr(num_legal),
                                                         batch_size, _ptr(feats), _stream(dev)),
                       "extract_fnn_features_batch")
        return feats

    def fnn_successor_features_batch(self, states: torch.Tensor, legal_moves: torch.Tensor,
                                     action_to_root: torch.Tensor, move_indices: torch.Tensor,
                                     num_actions: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, None, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, states.shape[0],
                            (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        action_to_root = _need(action_to_root, "action_to_root", torch.int64, num_actions)
        move_indices = _need(move_indices, "move_indices", torch.int64, num_actions)
        dev = states.device
        feats = torch.empty((num_actions, FNN_FEAT_DIM), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_fnn_successor_features(
                _ptr(states), states.shape[0], _ptr(legal_moves), _ptr(action_to_root), _ptr(move_indices),
                num_actions, _ptr(feats), _stream(dev)), "fnn_successor_features_batch")
        return feats

    def apply_moves_batch(self, states: torch.Tensor, moves: torch.Tensor, batch_size: int) -> None:
        if not states.is_contiguous():
            raise ValueError("states: must be contiguous (updated in place)")
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        moves = _need(moves, "moves", torch.uint8, batch_size, (SIZEOF_GPU_MOVE,))
        dev = states.device
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_apply_moves(_ptr(states), _ptr(moves), batch_size, _stream(dev)),
                       "apply_moves_batch")

    def check_results_batch(self, states: torch.Tensor, batch_size: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        out = torch.empty((batch_size,), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_check_results(_ptr(states), batch_size, _ptr(out), _stream(dev)),
                       "check_results_batch")
        return out

    def compute_centroids_batch(self, states: torch.Tensor, batch_size: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        out = torch.empty((batch_size, 2), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_compute_centroids(_ptr(states), batch_size, _ptr(out), _stream(dev)),
                       "compute_centroids_batch")
        return out

    def legal_moves_to_actions_batch(self, states: torch.Tensor, legal_moves: torch.Tensor,
                                     num_legal: torch.Tensor, batch_size: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, batch_size,
                            (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, batch_size)
        dev = states.device
        out = torch.empty((batch_size, MAX_LEGAL_MOVES), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_legal_moves_to_actions(_ptr(states), _ptr(legal_moves), _ptr(num_legal),
                                                           batch_size, _ptr(out), _stream(dev)),
                       "legal_moves_to_actions_batch")
        return out

    # -- inputs for benchmarks and tests --------------------------------------
    def generate_positions(self, seed: int, first_game: int, count: int, max_ply: int,
                           expansion_mask: int = 0, device: str | torch.device = "cuda") -> torch.Tensor:
        """Seeded random-playout positions (same recipe as the CPU oracle's generator)."""
        out = torch.empty((count, SIZEOF_HIVE_STATE), dtype=torch.uint8, device=device)
        with torch.cuda.device(out.device):
            _lib.check(self._lib.hv_generate_positions(seed, first_game, count, max_ply, expansion_mask,
                                                       _ptr(out), _stream(out.device)),
                       "generate_positions")
        return out

    def device_error_word(self, clear: bool = True) -> int:
        import ctypes
        v = ctypes.c_uint32(0)
        _lib.check(self._lib.hv_get_error(ctypes.addressof(v), int(clear)), "hv_get_error")
        return int(v.value)

    def __getattr__(self, name):
        if name in _OUT_OF_SCOPE:
            def _nope(*a, **k):
                raise NotImplementedError(f"{name} is outside the self-play hot path of this build")
            return _nope
        raise AttributeError(name)


_extension: HiveGPUExtension | None = None


def load_extension() -> HiveGPUExtension:
    """Same entry point as hive_gpu.load_extension() (hive_gpu/__init__.py:45-89)."""
    global _extension
    if _extension is None:
        _extension = HiveGPUExtension()
    return _extension
