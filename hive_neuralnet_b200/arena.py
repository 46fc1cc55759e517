"""Arena / match evaluation on the self-play kernels (reference arena.py).

Two searchers play a batch of games against each other: every step the
active games are split by which model is to move, each side searches its
rows (Gumbel-root MCTS with sequential halving, PUCT, or the raw policy) and
the chosen moves are written back into the shared state tensor.  The move
choosers, tree slicing and the score tally follow arena.py:149-231 and
:405-1180; checkpoints written by the reference load through
:func:`load_checkpoint`.

Differences from the reference:

* the PRS model line is outside the self-play path: ``model_type="prs"``
  raises ``NotImplementedError``;
* Gumbel noise and multinomial draws come from the orchestrator's CUDA
  generator (``config.seed``), not the global torch RNG;
* ``choose_fnn_puct_moves`` passes the evaluator's child Q to
  ``_expand_root_if_needed``: the reference call (arena.py:663-666) omits it
  and raises ``TypeError`` against the 8-argument method
  (fnn_puct_orchestrator.py:300);
* :func:`play_arena` returns the tally (and timing) instead of printing it;
  :func:`main` prints the reference's report.

Kept on purpose: when any row of a side's batch has an immediate win, the
rows without one play their first legal move (arena.py:458-460, 544-545);
the halving keeps ``max(1, max_alive // 2)`` slots by a batch-wide top-k,
so a row with fewer live candidates can take back padded slots
(arena.py:511-525).
"""
from __future__ import annotations

import argparse
import glob
import io
import math
import os
import pickle
import time
from dataclasses import dataclass
from typing import Literal

import numpy as np
import torch

from .fnn import FNNConfig, HiveFNN
from .hive_gpu import SIZEOF_GPU_MOVE, load_extension
from .hybrid import HiveHybridGNN, HybridGNNConfig
from .orchestrator import (FNNMCTSConfig, FNNMCTSOrchestrator, FNNPUCTConfig, FNNPUCTOrchestrator,
                           HybridMCTSConfig, HybridMCTSOrchestrator)

ModelType = Literal["fnn", "fnn_transformer", "prs"]
_OFF_TURN = 3412

FNN_DEFAULT_PATTERNS = (
    "checkpoints_fnn_small/hive_fnn_checkpoint_*.pt",
    "checkpoints_fnn_medium/hive_fnn_checkpoint_*.pt",
    "checkpoints_fnn_large/hive_fnn_checkpoint_*.pt",
    "checkpoints_fnn/hive_fnn_checkpoint_*.pt",
)
FNN_TRANSFORMER_DEFAULT_PATTERNS = (
    "checkpoints_fnn_transformer/hybrid_gnn_checkpoint_*.pt",
    "checkpoints_bootstrap_*_fnn_transformer_*/hybrid_gnn_checkpoint_*.pt",
)


def _no_prs() -> NotImplementedError:
    return NotImplementedError("the PRS model line is outside the self-play hot path of this build")


@dataclass
class ArenaMoveResult:
    chosen_slots: np.ndarray
    move_bytes: np.ndarray


# ---------------------------------------------------------------------------
# checkpoints and configuration (arena.py:84-231)
# ---------------------------------------------------------------------------
# Config classes pickled inside the reference's checkpoints, mapped to this
# package's classes with the same fields.
_CLASS_MAP = {
    ("hive_fnn.fnn_network", "FNNConfig"): FNNConfig,
    ("hive_fnn_transformer.fnn_transformer_net", "HybridGNNConfig"): HybridGNNConfig,
}


class _Unpickler(pickle.Unpickler):
    def find_class(self, module, name):
        hit = _CLASS_MAP.get((module, name))
        return hit if hit is not None else super().find_class(module, name)


class _PickleModule:
    Unpickler = _Unpickler
    __name__ = "hive_neuralnet_b200.arena._PickleModule"

    @staticmethod
    def load(f, **kw):
        return _Unpickler(f, **kw).load()


def read_checkpoint(path: str) -> dict:
    """A reference checkpoint dict (``net_config``, ``model_state_dict``, ...)
    with its config objects mapped onto this package's classes."""
    with open(path, "rb") as f:
        data = f.read()
    return torch.load(io.BytesIO(data), map_location="cpu", weights_only=False, pickle_module=_PickleModule)


def load_checkpoint(model_type: ModelType, path: str, device: str = "cuda") -> torch.nn.Module:
    """arena.py:124-146 for the FNN and FNN-transformer lines."""
    if model_type == "prs":
        raise _no_prs()
    ckpt = read_checkpoint(path)
    net = (HiveFNN(ckpt["net_config"]) if model_type == "fnn" else HiveHybridGNN(ckpt["net_config"]))
    net = net.to(device).eval()
    net.load_state_dict(ckpt["model_state_dict"])
    return net


def _latest_by_mtime(paths: list[str]) -> str | None:
    return max(paths, key=lambda p: (os.path.getmtime(p), p)) if paths else None


def latest_checkpoint(model_type: ModelType) -> str | None:
    if model_type == "prs":
        raise _no_prs()
    patterns = FNN_DEFAULT_PATTERNS if model_type == "fnn" else FNN_TRANSFORMER_DEFAULT_PATTERNS
    return _latest_by_mtime([p for pat in patterns for p in glob.glob(pat)])


def default_sims(model_type: ModelType) -> int:
    return 1024 if model_type in ("fnn", "fnn_transformer") else 256


def default_k(_: ModelType) -> int:
    return 16


def default_wave_size(model_type: ModelType) -> int:
    return 4 if model_type in ("fnn", "fnn_transformer") else 16


def parse_wave_schedule(spec: str | None) -> list[int] | None:
    if spec is None:
        return None
    parts = [p.strip() for p in spec.split(",") if p.strip()]
    return [max(1, int(p)) for p in parts] or None


def build_orchestrator(model_type: ModelType, net: torch.nn.Module, games: int, sims: int, k: int,
                       wave_parallel: bool, wave_size: int, expansion_mask: int, max_game_length: int,
                       temperature: float, temperature_drop_move: int, compile_forward: bool = False,
                       use_puct: bool = False, c_puct: float | None = None, root_q_min_visits: int | None = None,
                       eval_mode: bool = True, seed: int | None = None):
    """arena.py:149-231 (``compile_forward`` only concerned the PRS line)."""
    if model_type == "prs":
        raise _no_prs()
    if use_puct:
        if model_type == "fnn_transformer":
            raise ValueError("fnn_transformer arena currently supports only Gumbel root search")
        cfg = FNNPUCTConfig(num_simulations=sims, c_puct=c_puct if c_puct is not None else FNNPUCTConfig.c_puct,
                            temperature=temperature, temperature_drop_move=temperature_drop_move,
                            batch_size=games, max_game_length=max_game_length, expansion_mask=expansion_mask,
                            wave_size=wave_size, seed=seed)
        if eval_mode:
            cfg.dirichlet_epsilon = 0.0
            cfg.temperature_drop_move = 0
        return FNNPUCTOrchestrator(net, cfg), cfg
    cls = HybridMCTSConfig if model_type == "fnn_transformer" else FNNMCTSConfig
    cfg = cls(num_simulations=sims, max_num_considered_actions=k,
              c_puct=c_puct if c_puct is not None else FNNMCTSConfig.c_puct,
              root_q_min_visits=(int(root_q_min_visits) if root_q_min_visits is not None
                                 else FNNMCTSConfig.root_q_min_visits),
              temperature=temperature, temperature_drop_move=temperature_drop_move, batch_size=games,
              max_game_length=max_game_length, expansion_mask=expansion_mask, wave_parallel=wave_parallel,
              wave_size=wave_size, seed=seed)
    if eval_mode:
        cfg.dirichlet_epsilon = 0.0
        cfg.temperature_drop_move = 0
    orch = HybridMCTSOrchestrator(net, cfg) if model_type == "fnn_transformer" else FNNMCTSOrchestrator(net, cfg)
    return orch, cfg


# ---------------------------------------------------------------------------
# move choosers (arena.py:405-780)
# ---------------------------------------------------------------------------
def _empty(B: int) -> ArenaMoveResult:
    return ArenaMoveResult(np.zeros(B, np.int64), np.zeros((B, SIZEOF_GPU_MOVE), np.uint8))


def _gumbel(orch, B: int, L: int, scale: float) -> torch.Tensor:
    if scale > 0.0:
        u = torch.rand(B, L, device=orch.device, generator=orch.gen).clamp(1e-4, 1 - 1e-4)
        return -torch.log(-torch.log(u)) * scale
    return torch.zeros(B, L, dtype=torch.float32, device=orch.device)


def _visit_policy(visits: torch.Tensor, valid_slot: torch.Tensor) -> torch.Tensor:
    vf = visits.float()
    vsum = vf.sum(dim=1, keepdim=True)
    probs = torch.where(vsum > 0, vf / vsum.clamp(min=1.0), torch.zeros_like(vf))
    uni = valid_slot.float()
    uni = uni / uni.sum(dim=1, keepdim=True).clamp(min=1.0)
    return torch.where(vsum > 0, probs, uni)


def _pick(orch, probs, has_actions, move_numbers, stochastic, temperature_drop_move):
    """Greedy rows take the argmax, sampled rows (``stochastic`` before the
    temperature drop) draw from the normalised policy."""
    chosen = torch.zeros((probs.shape[0],), dtype=torch.int64, device=probs.device)
    if stochastic and move_numbers is not None:
        mn = torch.as_tensor(np.asarray(move_numbers), device=probs.device).to(torch.int64)
        sample = has_actions & (mn < temperature_drop_move)
    else:
        sample = torch.zeros_like(has_actions)
    greedy = has_actions & ~sample
    chosen = torch.where(greedy, probs.argmax(dim=1), chosen)
    if bool(sample.any().item()):
        sp = probs / probs.sum(dim=1, keepdim=True).clamp_min(1e-8)
        sp = torch.where(sample.unsqueeze(1), sp, torch.full_like(sp, 1.0))
        chosen = torch.where(sample, torch.multinomial(sp, 1, generator=orch.gen).squeeze(1), chosen)
    return chosen


def _result(chosen, legal_moves, num_legal, active_mask) -> ArenaMoveResult:
    """arena.py:561-570: inactive rows and rows without moves report slot 0 and
    zero bytes; an out-of-range choice falls back to slot 0."""
    B = legal_moves.shape[0]
    n = num_legal.to(torch.int64)
    act = torch.as_tensor(np.asarray(active_mask, dtype=bool), device=legal_moves.device)
    ok = act & (n > 0)
    slot = torch.where(ok & (chosen < n), chosen, torch.zeros_like(chosen))
    row = torch.arange(B, device=legal_moves.device)
    mb = torch.where(ok.unsqueeze(1), legal_moves[row, slot.clamp(max=legal_moves.shape[1] - 1)],
                     torch.zeros((B, SIZEOF_GPU_MOVE), dtype=torch.uint8, device=legal_moves.device))
    return ArenaMoveResult(slot.cpu().numpy(), mb.cpu().numpy())


def choose_fnn_moves(orch, states: torch.Tensor, active_mask: np.ndarray, tree=None, move_numbers=None,
                     stochastic: bool = False, gumbel_noise_scale: float = 0.0) -> ArenaMoveResult:
    """arena.py:405-570: Gumbel top-k at the root, rounds of root-mask PUCT
    simulations with sequential halving of the live slots, visit-count policy."""
    if isinstance(orch, FNNPUCTOrchestrator):
        return choose_fnn_puct_moves(orch, states, active_mask=active_mask, tree=tree, move_numbers=move_numbers,
                                     stochastic=stochastic)
    B = int(states.shape[0])
    cfg, dev, L = orch.config, orch.device, orch._max_legal
    if tree is None:
        tree = orch._alloc_tree(B)
    legal, nl, feats = orch.ext.generate_legal_moves_and_fnn_features_batch(states, B)
    n64 = nl.to(torch.int64)
    has_actions = torch.as_tensor(np.asarray(active_mask, dtype=bool), device=dev) & (n64 > 0)
    wins = orch._find_immediate_wins(states, legal, nl, B)
    has_win = wins >= 0
    max_n = int(n64.max().item()) if B > 0 else 0
    if max_n == 0:
        return _empty(B)
    max_k = min(int(cfg.max_num_considered_actions), max_n)
    priors, _, child_q = orch._eval_states(states, legal, nl, B, feats)
    any_win = bool(has_win.any().item())
    if any_win:
        rows_w = torch.nonzero(has_win).squeeze(1)
        priors.zero_()
        priors[rows_w, wins[rows_w]] = 1.0
        child_q.zero_()
    valid_slot = orch._slot_idx < n64.unsqueeze(1)
    legal_logits = torch.where(valid_slot, priors.clamp(min=1e-20).log(), torch.full_like(priors, -1e30))
    if orch.trace is not None:
        orch.trace.append(dict(kind="root", states=states.clone(), legal=legal.clone(), nl=nl.clone(),
                               priors=priors.clone(), child_q=child_q.clone(), any_win=any_win,
                               game_active=has_actions.to(torch.int8)))
    if any_win:
        chosen = torch.where(has_win, wins, torch.zeros_like(wins))
        return _result(chosen, legal, nl, active_mask)
    gumbel = torch.where(valid_slot, _gumbel(orch, B, L, gumbel_noise_scale), torch.full_like(priors, -1e30))
    top = torch.topk(gumbel + legal_logits, max_k, dim=1).indices
    active_i8 = has_actions.to(torch.int8)
    orch._expand_root_if_needed(tree, states, legal, nl, priors, child_q, active_i8, B)
    orch._apply_root_dirichlet(tree, B, has_actions)
    alive = torch.zeros(B, L, dtype=torch.int8, device=dev)
    alive.scatter_(1, top, 1)
    n_rounds = max(1, int(math.ceil(math.log2(max(max_k, 2)))))
    sims_per_round = max(1, int(cfg.num_simulations) // n_rounds)
    schedule = getattr(cfg, "wave_schedule", None)
    for r in range(n_rounds):
        if cfg.wave_parallel:
            W = schedule[min(r, len(schedule) - 1)] if schedule else cfg.wave_size
        else:
            W = 1
        if orch.trace is not None:
            orch.trace.append(dict(kind="round", alive=alive.clone(), sims=sims_per_round, W=W))
        orch._run_simulations(tree, states, active_i8, alive, B, sims_per_round, wave_size=W)
        cur_max = int(alive.sum(dim=1).max().item())
        if cur_max <= 1:
            continue
        num_keep = max(1, cur_max // 2)
        visits, q = orch._gather_root_child_stats(tree, B)
        sigma = (cfg.c_visit + int(visits.max().item())) * cfg.c_scale
        score = torch.where(alive.bool(), (gumbel + legal_logits + sigma * q).float(),
                            torch.full_like(priors, -1e30))
        keep = torch.topk(score, num_keep, dim=1).indices
        new_alive = torch.zeros_like(alive)
        new_alive.scatter_(1, keep, 1)
        alive = (new_alive * valid_slot.to(torch.int8)).contiguous()
    visits, _ = orch._gather_root_child_stats(tree, B)
    probs = _visit_policy(visits, valid_slot)
    if orch.trace is not None:
        orch.trace.append(dict(kind="searched", tree={k: v.clone() for k, v in tree.items()}, probs=probs.clone()))
    chosen = _pick(orch, probs, has_actions, move_numbers, stochastic, cfg.temperature_drop_move)
    return _result(chosen, legal, nl, active_mask)


def choose_fnn_policy_moves(orch, states: torch.Tensor, active_mask: np.ndarray, move_numbers=None,
                            stochastic: bool = False, gumbel_noise_scale: float = 0.0) -> ArenaMoveResult:
    """arena.py:573-623: the network's prior alone (no search)."""
    B = int(states.shape[0])
    cfg, L = orch.config, orch._max_legal
    legal, nl, feats = orch.ext.generate_legal_moves_and_fnn_features_batch(states, B)
    priors, _, _ = orch._eval_states(states, legal, nl, B, feats)
    n64 = nl.to(torch.int64)
    valid_slot = orch._slot_idx < n64.unsqueeze(1)
    legal_logits = torch.where(valid_slot, priors.clamp(min=1e-20).log(), torch.full_like(priors, -1e30))
    if gumbel_noise_scale > 0.0:
        scores = legal_logits + _gumbel(orch, B, L, gumbel_noise_scale)
    else:
        scores = torch.where(valid_slot, priors, torch.full_like(priors, -1.0))
    has_actions = torch.as_tensor(np.asarray(active_mask, dtype=bool), device=orch.device) & (n64 > 0)
    masked = torch.where(valid_slot, scores.float(), torch.full_like(scores, float("-inf")))
    chosen = torch.argmax(masked, dim=1)  # first maximum over the legal prefix
    if stochastic and move_numbers is not None:
        probs = (torch.softmax(masked, dim=1) if gumbel_noise_scale > 0.0
                 else torch.where(valid_slot, scores.float().clamp_min(0), torch.zeros_like(scores)))
        sampled = _pick(orch, probs, has_actions, move_numbers, True, cfg.temperature_drop_move)
        mn = torch.as_tensor(np.asarray(move_numbers), device=orch.device).to(torch.int64)
        chosen = torch.where(mn < cfg.temperature_drop_move, sampled, chosen)
    return _result(chosen, legal, nl, active_mask)


def choose_fnn_puct_moves(orch: FNNPUCTOrchestrator, states: torch.Tensor, active_mask: np.ndarray, tree=None,
                          move_numbers=None, stochastic: bool = False) -> ArenaMoveResult:
    """arena.py:626-729: PUCT over every legal root slot, visit-count policy."""
    B = int(states.shape[0])
    cfg, dev, L = orch.config, orch.device, orch._max_legal
    if tree is None:
        tree = orch._alloc_tree(B)
    legal, nl, feats = orch.ext.generate_legal_moves_and_fnn_features_batch(states, B)
    n64 = nl.to(torch.int64)
    has_actions = torch.as_tensor(np.asarray(active_mask, dtype=bool), device=dev) & (n64 > 0)
    wins = orch._find_immediate_wins(states, legal, nl, B)
    has_win = wins >= 0
    if (int(n64.max().item()) if B > 0 else 0) == 0:
        return _empty(B)
    priors, _, child_q = orch._eval_states(states, legal, nl, B, feats)
    any_win = bool(has_win.any().item())
    if any_win:
        rows_w = torch.nonzero(has_win).squeeze(1)
        priors.zero_()
        priors[rows_w, wins[rows_w]] = 1.0
    game_active = has_actions.to(torch.int8)
    orch._expand_root_if_needed(tree, states, legal, nl, priors, child_q, game_active, B)
    orch._apply_root_dirichlet(tree, B, has_actions)
    if any_win:
        chosen = torch.where(has_win, wins, torch.zeros_like(wins))
        return _result(chosen, legal, nl, active_mask)
    valid_slot = orch._slot_idx < n64.unsqueeze(1)
    orch._run_simulations(tree, states, game_active, valid_slot.to(torch.int8).contiguous(), B,
                          int(cfg.num_simulations))
    visits, _ = orch._gather_root_child_stats(tree, B)
    probs = _visit_policy(visits, valid_slot)
    chosen = _pick(orch, probs, has_actions, move_numbers, stochastic, cfg.temperature_drop_move)
    return _result(chosen, legal, nl, active_mask)


def choose_moves(model_type: ModelType, orch, states: torch.Tensor, active_mask: np.ndarray, tree=None,
                 move_numbers=None, stochastic: bool = False, gumbel_noise_scale: float = 0.0,
                 policy_only: bool = False) -> ArenaMoveResult:
    """arena.py:732-779"""
    if model_type == "prs":
        raise _no_prs()
    if policy_only:
        return choose_fnn_policy_moves(orch, states, active_mask=active_mask, move_numbers=move_numbers,
                                       stochastic=stochastic, gumbel_noise_scale=gumbel_noise_scale)
    return choose_fnn_moves(orch, states, active_mask=active_mask, tree=tree, move_numbers=move_numbers,
                            stochastic=stochastic, gumbel_noise_scale=gumbel_noise_scale)


# ---------------------------------------------------------------------------
# per-side tree rows (arena.py:782-903)
# ---------------------------------------------------------------------------
def _tree_child_nodes_from_slots(tree, chosen_slots: np.ndarray) -> np.ndarray:
    """Root child node of each chosen slot, -1 where the root has no such child."""
    B = int(chosen_slots.shape[0])
    dev = tree["root_node"].device
    row = torch.arange(B, device=dev)
    fc = tree["first_child"][row, tree["root_node"].long()]
    nc = tree["num_children"][row, tree["root_node"].long()]
    slot = torch.from_numpy(np.asarray(chosen_slots, dtype=np.int64)).to(dev)
    ok = (fc >= 0) & (slot >= 0) & (slot < nc)
    return torch.where(ok, fc.to(torch.int64) + slot, torch.full_like(slot, -1)).cpu().numpy()


def _reset_tree_rows(tree, rows: np.ndarray) -> None:
    if rows.size == 0:
        return
    r = torch.from_numpy(rows.astype(np.int64, copy=False)).to(tree["root_node"].device)
    for key, fill in (("visit_count", 0), ("total_value", 0.0), ("prior", 0.0), ("virtual_q_penalty", 0.0),
                      ("parent_idx", -1), ("move_bytes", 0), ("action_idx", -1), ("first_child", -1),
                      ("num_children", 0), ("is_terminal", 0), ("terminal_value", 0.0), ("node_count", 1),
                      ("root_node", 0), ("child_init_q", 0.0)):
        if key in tree:
            tree[key][r] = fill


def _slice_tree_rows(tree, rows: np.ndarray):
    if tree is None or rows.size == 0:
        return None
    r = torch.from_numpy(rows.astype(np.int64, copy=False)).to(tree["root_node"].device)
    return {k: v.index_select(0, r).clone() for k, v in tree.items()}


def _restore_tree_rows(tree, rows: np.ndarray, compact) -> None:
    if tree is None or compact is None or rows.size == 0:
        return
    r = torch.from_numpy(rows.astype(np.int64, copy=False)).to(tree["root_node"].device)
    for k, v in compact.items():
        tree[k].index_copy_(0, r, v)


def _run_side_rows(*, model_type: ModelType, orch, tree, states: torch.Tensor, rows: np.ndarray,
                   move_numbers: np.ndarray, stochastic: bool, gumbel_noise_scale: float,
                   policy_only: bool) -> None:
    """arena.py:858-903: search one side's rows, apply the moves, re-root."""
    if rows.size == 0:
        return
    r = torch.from_numpy(rows.astype(np.int64, copy=False)).to(states.device)
    sub = states.index_select(0, r).contiguous()
    sub_tree = _slice_tree_rows(tree, rows)
    sub_moves = move_numbers[rows].copy()
    res = choose_moves(model_type, orch, sub, active_mask=np.ones(rows.size, dtype=bool), tree=sub_tree,
                       move_numbers=sub_moves, stochastic=stochastic, gumbel_noise_scale=gumbel_noise_scale,
                       policy_only=policy_only)
    orch.ext.apply_moves_batch(sub, torch.from_numpy(res.move_bytes).to(states.device), int(rows.size))
    sub_moves += 1
    if sub_tree is not None:
        child = _tree_child_nodes_from_slots(sub_tree, res.chosen_slots)
        _reset_tree_rows(sub_tree, np.flatnonzero(child < 0))
        child_t = torch.from_numpy(child).to(states.device)
        orch._reroot_tree(sub_tree, child_t >= 0, child_t)
        _restore_tree_rows(tree, rows, sub_tree)
    states.index_copy_(0, r, sub)
    move_numbers[rows] = sub_moves


# ---------------------------------------------------------------------------
# the match loop and the tally (arena.py:1039-1180)
# ---------------------------------------------------------------------------
@dataclass
class ArenaResult:
    final_results: np.ndarray
    white_is_model_a: np.ndarray
    move_numbers: np.ndarray
    white_wins: int = 0
    black_wins: int = 0
    draws: int = 0
    capped: int = 0
    white_score: float = 0.0
    model_a_score: float = 0.0
    model_a_white_games: int = 0
    model_a_black_games: int = 0
    model_a_white_score: float = 0.0
    model_a_black_score: float = 0.0
    seconds: float = 0.0
    steps: int = 0


def tally(final_results: np.ndarray, white_is_model_a: np.ndarray) -> dict:
    """arena.py:1101-1151.  "white"/"black" name the two model slots (model A
    is the white slot); with alternating colours model A also plays black."""
    t = dict(white_wins=0, black_wins=0, draws=0, capped=0, white_score=0.0, model_a_score=0.0,
             model_a_white_games=0, model_a_black_games=0, model_a_white_score=0.0, model_a_black_score=0.0)
    for r, a_white in zip(np.asarray(final_results).tolist(), np.asarray(white_is_model_a).tolist()):
        side = "model_a_white" if a_white else "model_a_black"
        t[side + "_games"] += 1
        if r in (0, 3):
            t["capped"] += int(r == 0)
            t["draws"] += 1
            t["white_score"] += 0.5
            t["model_a_score"] += 0.5
            t[side + "_score"] += 0.5
        elif (r == 1 and a_white) or (r == 2 and not a_white):
            t["white_wins"] += 1
            t["white_score"] += 1.0
            t["model_a_score"] += 1.0
            t[side + "_score"] += 1.0
        else:
            t["black_wins"] += 1
    return t


def play_arena(white_model: ModelType, white_orch, black_model: ModelType, black_orch, games: int, *,
               expansion_mask: int = 7, max_game_length: int = 300, alternate_colors: bool = False,
               stochastic: bool = False, gumbel_noise_scale: float = 0.1, white_policy_only: bool = False,
               black_policy_only: bool = False, start_states: torch.Tensor | None = None) -> ArenaResult:
    """arena.py:1039-1099: play ``games`` games between the two searchers."""
    ext = load_extension()
    B = int(games)
    states = (start_states.to(white_orch.device).contiguous().clone() if start_states is not None
              else ext.create_initial_states(B, expansion_mask))
    trees = [white_orch._alloc_tree(B), black_orch._alloc_tree(B)]
    active = np.ones(B, dtype=bool)
    move_numbers = np.zeros(B, dtype=np.int32)
    white_is_model_a = np.zeros(B, dtype=bool)
    if alternate_colors:
        white_is_model_a[::2] = True
    else:
        white_is_model_a[: B // 2] = True
    torch.cuda.synchronize(states.device)
    t0 = time.perf_counter()
    steps = 0
    while bool(active.any()):
        turns = (states[:, _OFF_TURN].to(torch.int32) | (states[:, _OFF_TURN + 1].to(torch.int32) << 8)).cpu().numpy()
        white_turn = active & ((turns % 2 == 0) == white_is_model_a)
        black_turn = active & ~white_turn
        wr, br = np.flatnonzero(white_turn), np.flatnonzero(black_turn)
        _run_side_rows(model_type=white_model, orch=white_orch, tree=trees[0], states=states, rows=wr,
                       move_numbers=move_numbers, stochastic=stochastic, gumbel_noise_scale=gumbel_noise_scale,
                       policy_only=white_policy_only)
        _run_side_rows(model_type=black_model, orch=black_orch, tree=trees[1], states=states, rows=br,
                       move_numbers=move_numbers, stochastic=stochastic, gumbel_noise_scale=gumbel_noise_scale,
                       policy_only=black_policy_only)
        moved = np.concatenate([wr, br])
        if moved.size == 0:
            break
        mt = torch.from_numpy(moved.astype(np.int64)).to(states.device)
        res = ext.check_results_batch(states.index_select(0, mt).contiguous(), int(moved.size)).cpu().numpy()
        active[moved] = (res == 0) & (move_numbers[moved] < max_game_length)
        steps += 1
    final = ext.check_results_batch(states, B).cpu().numpy()
    seconds = time.perf_counter() - t0
    return ArenaResult(final_results=final, white_is_model_a=white_is_model_a, move_numbers=move_numbers.copy(),
                       seconds=seconds, steps=steps, **tally(final, white_is_model_a))


def main(argv: list[str] | None = None) -> None:
    """Command line of arena.py:906-1180 (FNN and FNN-transformer lines)."""
    ap = argparse.ArgumentParser(description="Arena: compare FNN / FNN-transformer checkpoints.")
    ap.add_argument("--white-model", choices=["fnn", "fnn_transformer", "prs"], default="fnn")
    ap.add_argument("--black-model", choices=["fnn", "fnn_transformer", "prs"], default="fnn")
    ap.add_argument("--white-checkpoint", type=str, default=None)
    ap.add_argument("--black-checkpoint", type=str, default=None)
    ap.add_argument("--games", type=int, default=50)
    for side in ("white", "black"):
        ap.add_argument(f"--{side}-sims", type=int, default=None)
        ap.add_argument(f"--{side}-k", type=int, default=None)
        ap.add_argument(f"--{side}-wave-size", type=int, default=None)
        ap.add_argument(f"--{side}-fnn-wave-schedule", type=str, default=None)
        ap.add_argument(f"--{side}-puct", action="store_true", default=False)
        ap.add_argument(f"--{side}-policy-only", action="store_true", default=False)
        ap.add_argument(f"--{side}-c-puct", type=float, default=None)
        ap.add_argument(f"--{side}-root-q-min-visits", type=int, default=None)
    ap.add_argument("--wave-parallel", action=argparse.BooleanOptionalAction, default=True)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--temperature-drop-move", type=int, default=20)
    ap.add_argument("--expansion-mask", type=int, default=7)
    ap.add_argument("--max-game-length", type=int, default=300)
    ap.add_argument("--alternate-colors", action="store_true")
    ap.add_argument("--stochastic", action="store_true")
    ap.add_argument("--gumbel-noise-scale", type=float, default=0.1)
    ap.add_argument("--compile-forward", action=argparse.BooleanOptionalAction, default=False)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    np.random.seed(args.seed)
    torch.manual_seed(args.seed)
    eval_mode = not args.stochastic
    sides = {}
    for side in ("white", "black"):
        model = getattr(args, f"{side}_model")
        path = getattr(args, f"{side}_checkpoint") or latest_checkpoint(model)
        if not path:
            raise SystemExit(f"No checkpoint found for {side} model type {model!r}")
        net = load_checkpoint(model, path)
        sims, k, ws = (getattr(args, f"{side}_{name}") for name in ("sims", "k", "wave_size"))
        sims = default_sims(model) if sims is None else sims
        k = default_k(model) if k is None else k
        ws = default_wave_size(model) if ws is None else ws
        orch, cfg = build_orchestrator(model, net, args.games, sims, k, args.wave_parallel, ws, args.expansion_mask,
                                       args.max_game_length, args.temperature, args.temperature_drop_move,
                                       args.compile_forward, use_puct=getattr(args, f"{side}_puct"),
                                       c_puct=getattr(args, f"{side}_c_puct"),
                                       root_q_min_visits=getattr(args, f"{side}_root_q_min_visits"),
                                       eval_mode=eval_mode, seed=args.seed + (0 if side == "white" else 1))
        cfg.wave_schedule = parse_wave_schedule(getattr(args, f"{side}_fnn_wave_schedule"))
        sides[side] = (model, path, orch, cfg, sims, k)
    (wm, wp, wo, wc, ws_, wk), (bm, bp, bo, bc, bs_, bk) = sides["white"], sides["black"]
    r = play_arena(wm, wo, bm, bo, args.games, expansion_mask=args.expansion_mask,
                   max_game_length=args.max_game_length, alternate_colors=args.alternate_colors,
                   stochastic=args.stochastic, gumbel_noise_scale=args.gumbel_noise_scale,
                   white_policy_only=args.white_policy_only, black_policy_only=args.black_policy_only)
    B = args.games
    print(f"White model:      {wm}\nWhite checkpoint: {wp}\nBlack model:      {bm}\nBlack checkpoint: {bp}")
    print(f"Arena config: games={B}, white_sims={ws_}, black_sims={bs_}, white_k={wk}, black_k={bk}, "
          f"white_root={'puct' if args.white_puct else 'gumbel'}, black_root={'puct' if args.black_puct else 'gumbel'}, "
          f"expansion_mask={args.expansion_mask}, max_game_length={args.max_game_length}, "
          f"stochastic={args.stochastic}, gumbel_noise_scale={args.gumbel_noise_scale}, "
          f"wave_parallel={args.wave_parallel}, alternate_colors={args.alternate_colors}")
    if args.alternate_colors:
        print(f"Model A score:    {r.model_a_score:.1f}/{B} = {r.model_a_score / B:.3f}")
        if r.model_a_white_games:
            print(f"Model A as white: {r.model_a_white_score:.1f}/{r.model_a_white_games} = "
                  f"{r.model_a_white_score / r.model_a_white_games:.3f}")
        if r.model_a_black_games:
            print(f"Model A as black: {r.model_a_black_score:.1f}/{r.model_a_black_games} = "
                  f"{r.model_a_black_score / r.model_a_black_games:.3f}")
    else:
        print(f"White wins:      {r.white_wins}\nBlack wins:      {r.black_wins}")
        print(f"Draws:           {r.draws}  (capped={r.capped})")
        print(f"White score:     {r.white_score:.1f}/{B} = {r.white_score / B:.3f}")
    print(f"Games/s:         {B / max(r.seconds, 1e-9):.3f}  ({r.steps} steps, {r.seconds:.1f} s)")


if __name__ == "__main__":
    main()
