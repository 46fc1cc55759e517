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
# device staging slots (and streams) of the chunked host-buffer pipeline
HOST_PIPELINE_STAGES = 3
# moves per position that the host-buffer pipeline sends over the host link
# as one pitched copy; the rest of each 256-move row is cleared on the host
# and the moves past this prefix are stored into the mapped host rows
HOST_MOVE_PREFIX = 64
# the row tails are cleared by torch's CPU threads; with fewer threads than
# this the clearing (about 300 MB per 262,144 positions) is slower than
# sending the tails over the link, and the whole rows are copied instead
HOST_CLEAR_MIN_THREADS = 8
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

    def generate_legal_moves_and_fnn_features_host(self, states: torch.Tensor, batch_size: int,
                                                   out: tuple | None = None, chunk: int = 32768,
                                                   device: torch.device | None = None,
                                                   move_prefix: int = HOST_MOVE_PREFIX):
        """Host-buffer form of :meth:`generate_legal_moves_and_fnn_features_batch`.

        ``states`` is a CPU uint8 ``[>=batch_size, 3424]`` tensor (pinned for
        overlap); results land in CPU tensors ``(moves [B,256,6] u8, num_legal
        [B] i32, features [B,122] f32)``, pinned when allocated here, or the
        caller's ``out`` triple.  The batch is cut into chunks that cycle
        through three streams and three device staging slots, so the
        host-to-device copy of one chunk, the kernel of the next and the
        device-to-host copy of a third overlap.  With pinned ``moves``, only
        the first ``move_prefix`` moves of each row cross the host link in
        one pitched copy, plus the moves of longer lists past it (stored
        into the mapped rows by a kernel); the calling thread clears the rest
        of each row in host memory meanwhile, so the zero padding (about
        half of the bytes returned) never crosses the link
        (``hv_download_moves``; with fewer than ``HOST_CLEAR_MIN_THREADS``
        torch threads the whole rows are copied).  Returns after queuing; the caller's current
        stream is ordered after every chunk, so
        ``torch.cuda.current_stream().synchronize()`` makes the outputs valid.
        """
        if not isinstance(states, torch.Tensor) or states.is_cuda or states.dtype != torch.uint8:
            raise ValueError("states: expected a CPU uint8 tensor")
        if states.dim() != 2 or states.shape[0] < batch_size or states.shape[1] != SIZEOF_HIVE_STATE:
            raise ValueError(f"states: expected [>= {batch_size}, {SIZEOF_HIVE_STATE}], got {tuple(states.shape)}")
        if not states.is_contiguous():
            raise ValueError("states: expected a contiguous tensor")
        if chunk <= 0:
            raise ValueError("chunk must be positive")
        if not 0 <= move_prefix <= MAX_LEGAL_MOVES or move_prefix % 8:
            raise ValueError("move_prefix: a multiple of 8 in 0..256")
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        if out is None:
            pin = states.is_pinned()
            out = (torch.empty((batch_size, MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE), dtype=torch.uint8, pin_memory=pin),
                   torch.empty((batch_size,), dtype=torch.int32, pin_memory=pin),
                   torch.empty((batch_size, FNN_FEAT_DIM), dtype=torch.float32, pin_memory=pin))
        h_moves, h_nl, h_feat = out
        for t, nm, dt, tail in ((h_moves, "moves", torch.uint8, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE)),
                                (h_nl, "num_legal", torch.int32, ()),
                                (h_feat, "features", torch.float32, (FNN_FEAT_DIM,))):
            if t.is_cuda or t.dtype != dt or t.shape[0] < batch_size or tuple(t.shape[1:]) != tail \
                    or not t.is_contiguous():
                raise ValueError(f"out {nm}: expected a contiguous CPU {dt} tensor [>= {batch_size}, {tail}]")
        chunk = min(chunk, max(batch_size, 1))
        # rows cleared on the host take the prefix download (hv_download_moves
        # falls back to one full copy for pageable memory or a misaligned row)
        split = (move_prefix < MAX_LEGAL_MOVES and h_moves.is_pinned() and h_moves.data_ptr() % 16 == 0
                 and torch.get_num_threads() >= HOST_CLEAR_MIN_THREADS)
        slots, streams = self._staging(dev, chunk)
        cur = torch.cuda.current_stream(dev)
        ready = cur.record_event()
        with torch.cuda.device(dev):
            for s in streams:
                s.wait_event(ready)
            for i, lo in enumerate(range(0, batch_size, chunk)):
                n = min(chunk, batch_size - lo)
                d_st, d_mv, d_nl, d_ft = slots[i % len(slots)]
                s = streams[i % len(streams)]
                with torch.cuda.stream(s):
                    # heights, bitboards and fields, and the stack levels over the
                    # rows that hold pieces (hv_stage_host_states)
                    _lib.check(self._lib.hv_stage_host_states(states.data_ptr() + lo * SIZEOF_HIVE_STATE, n,
                                                              _ptr(d_st), s.cuda_stream),
                               "generate_legal_moves_and_fnn_features_host")
                    _lib.check(self._lib.hv_generate_legal_moves_and_fnn_features(
                        _ptr(d_st), n, _ptr(d_mv), _ptr(d_nl), _ptr(d_ft), s.cuda_stream),
                        "generate_legal_moves_and_fnn_features_host")
                    if split:
                        # the row tails, on this thread while the device works;
                        # cleared before the download that may store into them
                        h_moves[lo:lo + n, move_prefix:].zero_()
                        _lib.check(self._lib.hv_download_moves(_ptr(d_mv), _ptr(d_nl), n,
                                                               h_moves.data_ptr() + lo * MAX_LEGAL_MOVES *
                                                               SIZEOF_GPU_MOVE, move_prefix, s.cuda_stream),
                                   "generate_legal_moves_and_fnn_features_host")
                    else:
                        h_moves[lo:lo + n].copy_(d_mv[:n], non_blocking=True)
                    h_nl[lo:lo + n].copy_(d_nl[:n], non_blocking=True)
                    h_feat[lo:lo + n].copy_(d_ft[:n], non_blocking=True)
            for s in streams:
                cur.wait_stream(s)
        return h_moves, h_nl, h_feat

    def _staging(self, dev: torch.device, chunk: int):
        """Three device staging slots and three streams per (device, chunk), kept for the process."""
        cache = self.__dict__.setdefault("_staging_cache", {})
        key = (dev.index, chunk)
        if key not in cache:
            with torch.cuda.device(dev):
                slots = [(torch.empty((chunk, SIZEOF_HIVE_STATE), dtype=torch.uint8, device=dev),
                          torch.empty((chunk, MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=dev),
                          torch.empty((chunk,), dtype=torch.int32, device=dev),
                          torch.empty((chunk, FNN_FEAT_DIM), dtype=torch.float32, device=dev))
                         for _ in range(HOST_PIPELINE_STAGES)]
                streams = [torch.cuda.Stream(dev) for _ in range(HOST_PIPELINE_STAGES)]
            cache[key] = (slots, streams)
        return cache[key]

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

    def queen_escape_flags_batch(self, states: torch.Tensor, batch_size: int) -> torch.Tensor:
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        out = torch.empty((batch_size,), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_queen_escape_flags(_ptr(states), batch_size, _ptr(out), _stream(dev)),
                       "queen_escape_flags_batch")
        return out

    def child_probe_batch(self, states: torch.Tensor, legal_moves: torch.Tensor, num_legal: torch.Tensor,
                          batch_size: int, want_escape: bool = False):
        """(results, queen_surround, queen_escape) of every legal child, [B, 256] each."""
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, batch_size, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, batch_size)
        dev = states.device
        res = torch.empty((batch_size, MAX_LEGAL_MOVES), dtype=torch.int32, device=dev)
        sur = torch.empty((batch_size, MAX_LEGAL_MOVES), dtype=torch.int32, device=dev)
        esc = torch.empty((batch_size, MAX_LEGAL_MOVES), dtype=torch.uint8, device=dev) if want_escape else None
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_child_probe(_ptr(states), _ptr(legal_moves), _ptr(num_legal), batch_size,
                                                int(want_escape), _ptr(res), _ptr(sur), _ptr(esc), _stream(dev)),
                       "child_probe")
        return res, sur, esc

    # -- hybrid transformer inputs (bindings.cpp:48-52, 78-81, 110-114) ------
    def _hybrid_tokens_out(self, B: int, dev):
        return (torch.empty((B, HYBRID_MAX_PIECE_TOKENS, HYBRID_NODE_FEAT_DIM), dtype=torch.float32, device=dev),
                torch.empty((B, HYBRID_MAX_PIECE_TOKENS), dtype=torch.int32, device=dev),
                torch.empty((B, HYBRID_MAX_PIECE_TOKENS), dtype=torch.int32, device=dev),
                torch.empty((B, HYBRID_MAX_PIECE_TOKENS), dtype=torch.int32, device=dev),
                torch.empty((B, HYBRID_MAX_PIECE_TOKENS), dtype=torch.bool, device=dev),
                torch.empty((B, HYBRID_GLOBAL_FEAT_DIM), dtype=torch.float32, device=dev),
                torch.empty((B,), dtype=torch.int32, device=dev))

    def hybrid_transformer_encode_with_moves_batch(self, states: torch.Tensor, legal_moves: torch.Tensor,
                                                   num_legal: torch.Tensor, batch_size: int):
        """(token_features [B,28,27], token_q, token_r, token_z [B,28] i32, token_mask [B,28] bool,
        global_features [B,6], num_tokens [B] i32); game_logic.cu:652-702."""
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        out = self._hybrid_tokens_out(batch_size, dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_hybrid_encode(_ptr(states), batch_size, *(_ptr(t) for t in out), _stream(dev)),
                       "hybrid_transformer_encode_with_moves_batch")
        return out

    def hybrid_transformer_move_features_batch(self, states: torch.Tensor, legal_moves: torch.Tensor,
                                               num_legal: torch.Tensor, batch_size: int) -> torch.Tensor:
        """[B, 256, 31] f32 move features; game_logic.cu:704-727."""
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, batch_size, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, batch_size)
        dev = states.device
        mf = torch.empty((batch_size, MAX_LEGAL_MOVES, HYBRID_MOVE_FEAT_DIM), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_hybrid_move_features(_ptr(states), _ptr(legal_moves), _ptr(num_legal),
                                                         batch_size, _ptr(mf), _stream(dev)),
                       "hybrid_transformer_move_features_batch")
        return mf

    def generate_legal_moves_and_hybrid_root_features_batch(self, states: torch.Tensor, batch_size: int):
        """(moves, num_legal, fnn_features, token_features, token_q, token_r, token_z, token_mask,
        global_features, move_features); game_logic.cu:1469-1535."""
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        dev = states.device
        moves = torch.empty((batch_size, MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=dev)
        num_legal = torch.empty((batch_size,), dtype=torch.int32, device=dev)
        feats = torch.empty((batch_size, FNN_FEAT_DIM), dtype=torch.float32, device=dev)
        tok = self._hybrid_tokens_out(batch_size, dev)
        mf = torch.empty((batch_size, MAX_LEGAL_MOVES, HYBRID_MOVE_FEAT_DIM), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_generate_legal_moves_and_hybrid_root_features(
                _ptr(states), batch_size, _ptr(moves), _ptr(num_legal), _ptr(feats), *(_ptr(t) for t in tok),
                _ptr(mf), _stream(dev)), "generate_legal_moves_and_hybrid_root_features_batch")
        return (moves, num_legal, feats) + tok[:6] + (mf,)

    def _legal_mask(self, states, moves, num_legal, batch_size):
        dev = states.device
        masks = torch.empty((batch_size, ACTION_SPACE_SIZE), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_legal_mask(_ptr(states), _ptr(moves), _ptr(num_legal), batch_size, _ptr(masks),
                                               _stream(dev)), "legal_mask")
        return masks

    def generate_legal_mask_batch(self, states: torch.Tensor, batch_size: int):
        """(masks [B, 85834] f32, num_legal [B] i32); game_logic.cu:737-769."""
        moves, num_legal = self.generate_legal_moves_batch(states, batch_size)
        return self._legal_mask(_need(states, "states", torch.uint8, batch_size), moves, num_legal,
                                batch_size), num_legal

    def generate_legal_moves_and_mask_batch(self, states: torch.Tensor, batch_size: int):
        """(moves [B,256,6] u8, num_legal [B] i32, masks [B, 85834] f32); game_logic.cu:782-809."""
        moves, num_legal = self.generate_legal_moves_batch(states, batch_size)
        return moves, num_legal, self._legal_mask(_need(states, "states", torch.uint8, batch_size), moves,
                                                  num_legal, batch_size)

    def root_tactical_probe_batch(self, states: torch.Tensor, legal_moves: torch.Tensor, num_legal: torch.Tensor,
                                  priors: torch.Tensor, batch_size: int, enable_win_in_one: bool = True,
                                  enable_check_opponent_wins: bool = True, enable_win_in_two: bool = True):
        """(winning_move [B] i64, allowed_slots [B,256] u8, forced_random [B] u8), game_logic.cu:1579-1615."""
        states = _need(states, "states", torch.uint8, batch_size, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, batch_size, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, batch_size)
        priors = _need(priors, "priors", torch.float32, batch_size, (MAX_LEGAL_MOVES,))
        dev = states.device
        win = torch.empty((batch_size,), dtype=torch.int64, device=dev)
        allowed = torch.empty((batch_size, MAX_LEGAL_MOVES), dtype=torch.uint8, device=dev)
        forced = torch.empty((batch_size,), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_root_tactical_probe(
                _ptr(states), _ptr(legal_moves), _ptr(num_legal), _ptr(priors), batch_size,
                int(bool(enable_win_in_one)), int(bool(enable_check_opponent_wins)), int(bool(enable_win_in_two)),
                _ptr(win), _ptr(allowed), _ptr(forced), _stream(dev)), "root_tactical_probe_batch")
        return win, allowed, forced

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

    # -- MCTS tree (bindings.cpp:110-226) ------------------------------------
    # Tree tensors in binding order: (vc i32, tv f32, pr f32, pa i32, vq f32,
    # mb u8[...,6], ai i32, fc i32, nc i32, it i8, tv2 f32, cnt i32[B]).
    _TREE_DTYPES = (torch.int32, torch.float32, torch.float32, torch.int32, torch.float32, torch.uint8,
                    torch.int32, torch.int32, torch.int32, torch.int8, torch.float32, torch.int32)

    def _tree(self, tensors, max_nodes: int, B: int) -> "_lib.HvTree":
        if len(tensors) != 12:
            raise ValueError(f"expected 12 tree tensors, got {len(tensors)}")
        for i, (t, dt) in enumerate(zip(tensors, self._TREE_DTYPES)):
            if not isinstance(t, torch.Tensor) or t.dtype != dt or not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"tree tensor {i}: expected contiguous CUDA {dt}")
            need = B if i == 11 else B * max_nodes * (6 if i == 5 else 1)
            if t.numel() < need:
                raise ValueError(f"tree tensor {i}: {t.numel()} elements < {need} for B={B}, max_nodes={max_nodes}")
        return _lib.HvTree(*[t.data_ptr() for t in tensors], int(max_nodes))

    def _select(self, tree, mode, child_init_q, game_active, root_nodes, alive_mask, root_slots,
                num_candidates, max_root_children, c_puct, B, W, max_nodes, det, sigma, q_penalty):
        import ctypes
        dev = tree[0].device
        total = W * num_candidates * B if mode == 2 else W * B
        leaf = torch.zeros((total,), dtype=torch.int32, device=dev)
        paths = torch.zeros((total, MAX_TREE_DEPTH, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=dev)
        plen = torch.zeros((total,), dtype=torch.int32, device=dev)
        vlp = torch.zeros((total, MAX_TREE_DEPTH), dtype=torch.int32, device=dev)
        vll = torch.zeros((total,), dtype=torch.int32, device=dev)
        ts = self._tree(tree, max_nodes, B)
        game_active = _need(game_active, "game_active", torch.int8, B)
        root_nodes = _need(root_nodes, "root_nodes", torch.int32, B)
        if alive_mask is not None:
            alive_mask = _need(alive_mask, "alive_mask", torch.int8, B)
        if root_slots is not None:
            root_slots = _need(root_slots, "root_slots", torch.int32, B)
        if child_init_q is not None:
            child_init_q = _need(child_init_q, "child_init_q", torch.float32, B)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_select(
                ctypes.byref(ts), mode, _ptr(child_init_q), _ptr(game_active), _ptr(root_nodes),
                _ptr(alive_mask), _ptr(root_slots), num_candidates, max_root_children, float(c_puct), B, W,
                int(bool(det)), float(sigma), float(q_penalty), _ptr(leaf), _ptr(paths), _ptr(plen),
                _ptr(vlp), _ptr(vll), _stream(dev)), "mcts_select")
        return leaf, paths, plen, vlp, vll

    def mcts_select_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, game_active, root_nodes,
                          c_puct, B, W, max_nodes):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        return self._select(tree, 0, None, game_active, root_nodes, None, None, 1, MAX_LEGAL_MOVES, c_puct,
                            B, W, max_nodes, False, 4.0, 0.0)

    def mcts_select_with_root_mask_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt,
                                         child_init_q, game_active, root_nodes, alive_mask, max_root_children,
                                         c_puct, B, W, max_nodes, deterministic_non_root=False,
                                         non_root_sigma=4.0, q_penalty=0.0):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        return self._select(tree, 1, child_init_q, game_active, root_nodes, alive_mask, None, 1,
                            max_root_children, c_puct, B, W, max_nodes, deterministic_non_root,
                            non_root_sigma, q_penalty)

    def mcts_select_with_root_slots_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt,
                                          child_init_q, game_active, root_nodes, root_slots, num_candidates,
                                          max_root_children, c_puct, B, W, max_nodes,
                                          deterministic_non_root=False, non_root_sigma=4.0, q_penalty=0.0):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        return self._select(tree, 2, child_init_q, game_active, root_nodes, None, root_slots, num_candidates,
                            max_root_children, c_puct, B, W, max_nodes, deterministic_non_root,
                            non_root_sigma, q_penalty)

    def mcts_replay_batch(self, root_states, leaf_states, move_paths, path_lengths, leaf_indices, B, total):
        root_states = _need(root_states, "root_states", torch.uint8, B, (SIZEOF_HIVE_STATE,))
        if not leaf_states.is_contiguous() or leaf_states.dtype != torch.uint8 or leaf_states.shape[0] < total:
            raise ValueError("leaf_states: expected contiguous uint8 [total, 3424] (written in place)")
        move_paths = _need(move_paths, "move_paths", torch.uint8, total)
        path_lengths = _need(path_lengths, "path_lengths", torch.int32, total)
        leaf_indices = _need(leaf_indices, "leaf_indices", torch.int32, total)
        dev = root_states.device
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_replay(_ptr(root_states), _ptr(leaf_states), _ptr(move_paths),
                                                _ptr(path_lengths), _ptr(leaf_indices), B, total, _stream(dev)),
                       "mcts_replay")

    def _expand(self, tree, dense, backprop, child_init_q, child_q, leaf_indices, leaf_states, legal_moves,
                num_legal, priors, results, values, vl_paths, vl_lengths, B, total, max_nodes, q_penalty,
                want_was):
        import ctypes
        dev = tree[0].device
        ts = self._tree(tree, max_nodes, B)
        leaf_indices = _need(leaf_indices, "leaf_indices", torch.int32, total)
        leaf_states = _need(leaf_states, "leaf_states", torch.uint8, total, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, total, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, total)
        priors = _need(priors, "priors", torch.float32, total,
                       (MAX_LEGAL_MOVES,) if dense else (ACTION_SPACE_SIZE,))
        results = _need(results, "results", torch.int32, total)
        if dense:
            child_q = _need(child_q, "child_q_values", torch.float32, total, (MAX_LEGAL_MOVES,))
            child_init_q = _need(child_init_q, "child_init_q", torch.float32, B)
        if backprop:
            values = _need(values.reshape(-1), "nn_values", torch.float32, total)
            vl_paths = _need(vl_paths, "vl_paths", torch.int32, total)
            vl_lengths = _need(vl_lengths, "vl_lengths", torch.int32, total)
        was = torch.zeros((total,), dtype=torch.int8, device=dev) if want_was else None
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_expand(
                ctypes.byref(ts), int(dense), int(backprop), _ptr(child_init_q), _ptr(child_q),
                _ptr(leaf_indices), _ptr(leaf_states), _ptr(legal_moves), _ptr(num_legal), _ptr(priors),
                _ptr(results), _ptr(values), _ptr(vl_paths), _ptr(vl_lengths), _ptr(was), float(q_penalty),
                B, total, _stream(dev)), "mcts_expand")
        return was

    def mcts_expand_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, leaf_indices, leaf_states,
                          legal_moves, num_legal, action_probs, results, B, total, max_nodes):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        return self._expand(tree, False, False, None, None, leaf_indices, leaf_states, legal_moves, num_legal,
                            action_probs, results, None, None, None, B, total, max_nodes, 0.0, True)

    def mcts_expand_and_backprop_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, leaf_indices,
                                       leaf_states, legal_moves, num_legal, action_probs, results, nn_values,
                                       vl_paths, vl_lengths, B, total, max_nodes):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        self._expand(tree, False, True, None, None, leaf_indices, leaf_states, legal_moves, num_legal,
                     action_probs, results, nn_values, vl_paths, vl_lengths, B, total, max_nodes, 0.0, False)

    def mcts_expand_dense_priors_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, child_init_q,
                                       child_q_values, leaf_indices, leaf_states, legal_moves, num_legal,
                                       priors_per_legal, results, B, total, max_nodes):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        return self._expand(tree, True, False, child_init_q, child_q_values, leaf_indices, leaf_states,
                            legal_moves, num_legal, priors_per_legal, results, None, None, None, B, total,
                            max_nodes, 0.0, True)

    def mcts_expand_and_backprop_dense_priors_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt,
                                                    child_init_q, child_q_values, leaf_indices, leaf_states,
                                                    legal_moves, num_legal, priors_per_legal, results,
                                                    nn_values, vl_paths, vl_lengths, B, total, max_nodes,
                                                    q_penalty=0.0):
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        self._expand(tree, True, True, child_init_q, child_q_values, leaf_indices, leaf_states, legal_moves,
                     num_legal, priors_per_legal, results, nn_values, vl_paths, vl_lengths, B, total, max_nodes,
                     q_penalty, False)

    def mcts_expand_and_backprop_dense_priors_slots_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt,
                                                          child_init_q, child_q_values, leaf_indices, leaf_states,
                                                          legal_moves, num_legal, priors_per_legal, results,
                                                          nn_values, vl_paths, vl_lengths, root_nodes, root_slots,
                                                          num_candidates, B, total, max_nodes, q_penalty=0.0):
        """mcts_expand_and_backprop_dense_priors_batch for the simulations of
        one select with the same root_nodes: mcts_select_with_root_slots_batch
        (its root_slots and num_candidates) or, with root_slots None,
        mcts_select_batch / mcts_select_with_root_mask_batch.  The same tree;
        the subtrees below different candidates / root children are updated
        in parallel (hv_mcts_expand_slots)."""
        import ctypes
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        dev = vc.device
        ts = self._tree(tree, max_nodes, B)
        leaf_indices = _need(leaf_indices, "leaf_indices", torch.int32, total)
        leaf_states = _need(leaf_states, "leaf_states", torch.uint8, total, (SIZEOF_HIVE_STATE,))
        legal_moves = _need(legal_moves, "legal_moves", torch.uint8, total, (MAX_LEGAL_MOVES, SIZEOF_GPU_MOVE))
        num_legal = _need(num_legal, "num_legal", torch.int32, total)
        priors = _need(priors_per_legal, "priors", torch.float32, total, (MAX_LEGAL_MOVES,))
        results = _need(results, "results", torch.int32, total)
        child_q = _need(child_q_values, "child_q_values", torch.float32, total, (MAX_LEGAL_MOVES,))
        child_init_q = _need(child_init_q, "child_init_q", torch.float32, B)
        values = _need(nn_values.reshape(-1), "nn_values", torch.float32, total)
        vl_paths = _need(vl_paths, "vl_paths", torch.int32, total)
        vl_lengths = _need(vl_lengths, "vl_lengths", torch.int32, total)
        root_nodes = _need(root_nodes, "root_nodes", torch.int32, B)
        if root_slots is not None:
            root_slots = _need(root_slots.to(torch.int32), "root_slots", torch.int32, B)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_expand_slots(
                ctypes.byref(ts), _ptr(child_init_q), _ptr(child_q), _ptr(leaf_indices), _ptr(leaf_states),
                _ptr(legal_moves), _ptr(num_legal), _ptr(priors), _ptr(results), _ptr(values), _ptr(vl_paths),
                _ptr(vl_lengths), _ptr(root_nodes), _ptr(root_slots), int(num_candidates), float(q_penalty), B,
                total, _stream(dev)), "mcts_expand_slots")

    def mcts_backprop_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, leaf_indices, nn_values,
                            vl_paths, vl_lengths, was_expanded, B, total, max_nodes):
        import ctypes
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        ts = self._tree(tree, max_nodes, B)
        dev = vc.device
        leaf_indices = _need(leaf_indices, "leaf_indices", torch.int32, total)
        nn_values = _need(nn_values.reshape(-1), "nn_values", torch.float32, total)
        vl_paths = _need(vl_paths, "vl_paths", torch.int32, total)
        vl_lengths = _need(vl_lengths, "vl_lengths", torch.int32, total)
        was_expanded = _need(was_expanded, "was_expanded", torch.int8, total)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_backprop(ctypes.byref(ts), _ptr(leaf_indices), _ptr(nn_values),
                                                  _ptr(vl_paths), _ptr(vl_lengths), _ptr(was_expanded), B, total,
                                                  _stream(dev)), "mcts_backprop")

    def mcts_extract_policy_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, move_numbers,
                                  root_nodes, temperature, temp_drop_move, pruning_threshold, B, max_nodes):
        import ctypes
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        ts = self._tree(tree, max_nodes, B)
        dev = vc.device
        move_numbers = _need(move_numbers.to(torch.int32), "move_numbers", torch.int32, B)
        root_nodes = _need(root_nodes, "root_nodes", torch.int32, B)
        pol = torch.zeros((B, ACTION_SPACE_SIZE), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_extract_policy(ctypes.byref(ts), _ptr(pol), _ptr(move_numbers),
                                                        _ptr(root_nodes), float(temperature), int(temp_drop_move),
                                                        float(pruning_threshold), B, _stream(dev)),
                       "mcts_extract_policy")
        return pol

    def mcts_apply_root_noise(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, noise, root_nodes,
                              max_children_pad, dir_eps, root_policy_temp, B, max_nodes):
        import ctypes
        tree = (vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt)
        ts = self._tree(tree, max_nodes, B)
        dev = vc.device
        noise = _need(noise, "noise", torch.float32, B)
        root_nodes = _need(root_nodes, "root_nodes", torch.int32, B)
        with torch.cuda.device(dev):
            _lib.check(self._lib.hv_mcts_root_noise(ctypes.byref(ts), _ptr(noise), _ptr(root_nodes),
                                                    int(max_children_pad), float(dir_eps), float(root_policy_temp),
                                                    B, _stream(dev)), "mcts_apply_root_noise")

    def mcts_select_replay_legal_fnn_root_slots_batch(self, vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt,
                                                      child_init_q, root_states, game_active, root_nodes,
                                                      root_slots, num_candidates, max_root_children, c_puct, B, W,
                                                      max_nodes, deterministic_non_root=False, non_root_sigma=4.0,
                                                      q_penalty=0.0):
        """Fused prefix of one Gumbel wave (game_logic.cu:1184-1254): root-slot
        select, replay, result check, legal moves + FNN features of the leaves."""
        leaf, paths, plen, vlp, vll = self.mcts_select_with_root_slots_batch(
            vc, tv, pr, pa, vq, mb, ai, fc, nc, it, tv2, cnt, child_init_q, game_active, root_nodes, root_slots,
            num_candidates, max_root_children, c_puct, B, W, max_nodes, deterministic_non_root, non_root_sigma,
            q_penalty)
        total = leaf.shape[0]
        # every row is written by the replay (zeros where a slot holds no simulation)
        leaf_states = torch.empty((total, SIZEOF_HIVE_STATE), dtype=torch.uint8, device=leaf.device)
        self.mcts_replay_batch(root_states, leaf_states, paths, plen, leaf, B, total)
        results = self.check_results_batch(leaf_states, total)
        legal, num_legal, feats = self.generate_legal_moves_and_fnn_features_batch(leaf_states, total)
        return leaf, leaf_states, legal, num_legal, feats, results, vlp, vll

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
