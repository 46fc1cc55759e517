"""Training-side inputs built with the self-play kernels.

``build_forward_batch`` is the reference trainer's
``FNNTrainer._build_forward_batch`` (hive_fnn/fnn_trainer.py:531-580): root
features, every successor's features, the successor -> root map and the
action counts of a replay batch, ready for a differentiable torch forward of
``HiveFNN`` (training keeps autograd in torch; only the inputs come from the
kernels).  ``build_hybrid_forward_batch`` adds the hybrid network's piece
tokens and per-move features (the replay buffer's cached bundle,
hive_fnn/fnn_replay_buffer.py:405-466).
"""
from __future__ import annotations

import torch

from .hive_gpu import load_extension
from .hybrid import HybridPieceTensorBatch


def _successor_index(num_actions: torch.Tensor, max_legal: int):
    slot = torch.arange(max_legal, device=num_actions.device, dtype=torch.int64).unsqueeze(0)
    valid = slot < num_actions.unsqueeze(1)
    rows = torch.arange(num_actions.shape[0], device=num_actions.device, dtype=torch.int64)
    return rows.unsqueeze(1).expand_as(valid)[valid], slot.expand_as(valid)[valid], valid


def build_forward_batch(state_bytes: torch.Tensor, batch_size: int, num_actions: torch.Tensor | None = None,
                        cached_root_features: torch.Tensor | None = None,
                        cached_legal_moves: torch.Tensor | None = None):
    """(root_features [B,122], successor_features [N,122], action_to_root [N] i64, num_actions [B] i64)."""
    ext = load_extension()
    if cached_root_features is not None and cached_legal_moves is not None:
        if num_actions is None:
            raise ValueError("Cached legal moves require cached action counts")
        root_features, legal_moves = cached_root_features.float(), cached_legal_moves
        num_actions = num_actions.to(torch.int64)
    else:
        legal_moves, num_legal, root_features = ext.generate_legal_moves_and_fnn_features_batch(state_bytes,
                                                                                                batch_size)
        num_actions = num_legal.to(torch.int64)
    action_to_root, move_indices, _ = _successor_index(num_actions, legal_moves.shape[1])
    total = int(action_to_root.shape[0])
    if total == 0:
        return root_features, root_features[:0], action_to_root, num_actions
    succ = ext.fnn_successor_features_batch(state_bytes, legal_moves.contiguous(), action_to_root, move_indices,
                                            total)
    return root_features, succ, action_to_root, num_actions


def build_hybrid_forward_batch(state_bytes: torch.Tensor, batch_size: int):
    """Inputs of ``HiveHybridGNN.forward`` for a batch of states: (root_features,
    successor_features, action_to_root, num_actions, piece_batch, move_features [N,31])."""
    ext = load_extension()
    (legal, num_legal, root_features, tf, tq, tr, tz, tm, gf,
     move_features) = ext.generate_legal_moves_and_hybrid_root_features_batch(state_bytes, batch_size)
    num_actions = num_legal.to(torch.int64)
    action_to_root, move_indices, valid = _successor_index(num_actions, legal.shape[1])
    total = int(action_to_root.shape[0])
    succ = (ext.fnn_successor_features_batch(state_bytes, legal, action_to_root, move_indices, total) if total
            else root_features[:0])
    pb = HybridPieceTensorBatch(tf, tq, tr, tz, tm, gf, tm.sum(dim=1, dtype=torch.int32))
    return root_features, succ, action_to_root, num_actions, pb, move_features[valid]
